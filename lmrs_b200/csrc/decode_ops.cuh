// decode_ops.cuh — the kernels around the quantized linears in a decode step.
//
//   * rmsnorm_kernel: residual += delta (optional), out = rmsnorm(residual) * w,
//     one rounding to the I/O type (reference: kernels/ffi/norm_ffi.cu:9-31);
//     FP8 form writes the e4m3 bytes and per-row scale of that rounded output
//     instead (bit-identical to rmsnorm -> fp8_quant_rows).
//   * rope_kv_kernel: rotate-half RoPE on q and k of the merged qkv row
//     (reference: kernels/ffi/pos_embed_ffi.cu:9-29), q to its buffer, k and v
//     into the paged KV cache at the step's position.
//   * silu_mul_kernel: out = silu(gate) * up from the merged gate|up row
//     (reference: kernels/ops/activation_kernels.cuh:40-48); FP8 form as above.
//   * decode_attn_kernel: one decode query per sequence against a paged KV
//     cache laid out as the reference's paged_attention_v1
//     (kernels/attention/paged_attention.cuh:14-108: cache[block][kv_head]
//     [block_offset][head_size], block table per sequence), GQA with the q heads
//     of one KV head in one CTA: S = Q K^T and O += P V on mma.sync (16 q-head
//     rows, 16 positions per warp step, fp32 accumulate), online softmax,
//     split over the context; up to 8 splits of one (sequence, KV head) form a
//     thread-block cluster and merge their (O, m, l) partials in split order
//     through distributed shared memory; with more splits (small batches) the
//     clusters' merged partials meet in a global workspace, merged there by
//     the last cluster to arrive (no second kernel).
// All are launched with programmatic dependent launch and call pdl_wait before
// touching their inputs.
#pragma once
#include <cooperative_groups.h>
#include "fp8_kernels.cuh"
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kNormThreads = 256;     // smallest CTA of the row kernels
constexpr int kRowMaxThreads = 1024;
constexpr int kRowMaxVecs = 4;        // 8-element vectors per thread held in registers

// Sum / max over the CTA (any multiple of 32 threads up to 1024).
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w];
  __syncthreads();
  return s;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

// 8 rounded activations -> 8 e4m3 bytes with the row scale s (same arithmetic
// as fp8_quant_rows_kernel: x / s rounded to nearest even, saturating).
__device__ __forceinline__ uint2 e4m3x8(const float (&v)[8], float s) {
  uint32_t out[2] = {0u, 0u};
  if (s != 0.f) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 pr = make_float2(__fdiv_rn(v[2 * i], s), __fdiv_rn(v[2 * i + 1], s));
      const uint32_t b =
          static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(pr, __NV_SATFINITE, __NV_E4M3));
      out[i >> 1] |= b << ((i & 1) * 16);
    }
  }
  return make_uint2(out[0], out[1]);
}

// Two packed T values <-> two floats.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  T e[2];
  *reinterpret_cast<uint32_t*>(e) = u;
  return make_float2(Act<T>::to_float(e[0]), Act<T>::to_float(e[1]));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  T e[2] = {Act<T>::from_float(a), Act<T>::from_float(b)};
  return *reinterpret_cast<uint32_t*>(e);
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Act<T>::to_float(e[i]);
}

// residual (+)= delta, out = rmsnorm(residual) * w, one CTA per row.  Thread t
// holds vectors v*blockDim + t (8 columns each, H % 8 == 0) of the row in
// registers: one read pass, one write pass.  FP8: out is replaced by the
// row's e4m3 bytes and scale, computed from the same rounded outputs.
template <typename T, bool FP8, int VPT>
__global__ void __launch_bounds__(kRowMaxThreads) rmsnorm_kernel(
    T* __restrict__ out, uint8_t* __restrict__ qout, float* __restrict__ qscale,
    T* __restrict__ resid, const T* __restrict__ delta, const T* __restrict__ w, int H, float eps) {
  // the norm weight is constant: read before the previous kernel has finished
  uint4 wv[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = (v * blockDim.x + threadIdx.x) * 8;
    wv[v] = c < H ? __ldg(reinterpret_cast<const uint4*>(w + c)) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int row = blockIdx.x;
  T* xr = resid + static_cast<int64_t>(row) * H;
  float x[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = (v * blockDim.x + threadIdx.x) * 8;
    if (c < H) {
      uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
      if (delta != nullptr) {
        const uint4 dv = *reinterpret_cast<const uint4*>(delta + static_cast<int64_t>(row) * H + c);
        const T* e = reinterpret_cast<const T*>(&xv);
        const T* de = reinterpret_cast<const T*>(&dv);
        uint4 sv;
        T* se = reinterpret_cast<T*>(&sv);
#pragma unroll
        for (int i = 0; i < 8; ++i) se[i] = Act<T>::from_float(Act<T>::to_float(e[i]) + Act<T>::to_float(de[i]));
        *reinterpret_cast<uint4*>(xr + c) = sv;  // the updated residual stream
        xv = sv;
      }
      unpack8<T>(xv, x[v]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += x[v][i] * x[v][i];
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / H + eps);
  float amax = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = (v * blockDim.x + threadIdx.x) * 8;
    if (c < H) {
      float wf[8];
      unpack8<T>(wv[v], wf);
      uint4 pk;
      T* oe = reinterpret_cast<T*>(&pk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        oe[i] = Act<T>::from_float(x[v][i] * inv * wf[i]);
        x[v][i] = Act<T>::to_float(oe[i]);
        amax = fmaxf(amax, fabsf(x[v][i]));
      }
      if (!FP8) *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * H + c) = pk;
    }
  }
  if (!FP8) return;
  const float sc = __fdiv_rn(block_max(amax, red), 448.0f);
  if (threadIdx.x == 0) qscale[row] = sc;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = (v * blockDim.x + threadIdx.x) * 8;
    if (c < H) *reinterpret_cast<uint2*>(qout + static_cast<int64_t>(row) * H + c) = e4m3x8(x[v], sc);
  }
}

// out[r, i] = silu(gu[r, i]) * gu[r, I + i]  (I = inter, I % 8 == 0).  Plain
// form: CTA (row, chunk), one vector per thread (gridDim.y chunks per row).
// FP8 form: one CTA per row with the row's VPT vectors per thread in
// registers (row absmax, then e4m3 from the same rounded values).
template <typename T, bool FP8, int VPT>
__global__ void __launch_bounds__(kRowMaxThreads) silu_mul_kernel(
    T* __restrict__ out, uint8_t* __restrict__ qout, float* __restrict__ qscale,
    const T* __restrict__ gu, int I) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int base = blockIdx.y * blockDim.x * 8 * VPT;
  const T* gr = gu + static_cast<int64_t>(row) * 2 * I;
  float y[VPT][8];
  float amax = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = base + (v * blockDim.x + threadIdx.x) * 8;
    if (c < I) {
      float g[8], u[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(gr + c), g);
      unpack8<T>(*reinterpret_cast<const uint4*>(gr + I + c), u);
      uint4 pk;
      T* oe = reinterpret_cast<T*>(&pk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        oe[i] = Act<T>::from_float((g[i] / (1.0f + expf(-g[i]))) * u[i]);
        y[v][i] = Act<T>::to_float(oe[i]);
        amax = fmaxf(amax, fabsf(y[v][i]));
      }
      if (!FP8) *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * I + c) = pk;
    }
  }
  if (!FP8) return;
  const float sc = __fdiv_rn(block_max(amax, red), 448.0f);
  if (threadIdx.x == 0) qscale[row] = sc;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = (v * blockDim.x + threadIdx.x) * 8;
    if (c < I) *reinterpret_cast<uint2*>(qout + static_cast<int64_t>(row) * I + c) = e4m3x8(y[v], sc);
  }
}

// FP8 silu * up for long rows: a cluster of C CTAs per row (grid (rows, C)),
// each CTA VPT vectors per thread of its column chunk in registers; the row
// absmax is exchanged through distributed shared memory (every CTA stores its
// maximum into slot [rank] of every CTA, then one cluster barrier).
constexpr int kSiluClusterThreads = 256;
constexpr int kSiluClusterVecs = 4;
constexpr int kSiluMaxCluster = 8;

template <typename T>
__global__ void __launch_bounds__(kSiluClusterThreads) silu_mul_fp8_cluster_kernel(
    uint8_t* __restrict__ qout, float* __restrict__ qscale, const T* __restrict__ gu, int I) {
  constexpr int VPT = kSiluClusterVecs;
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ float slot[kSiluMaxCluster];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.x;
  const int base = rank * kSiluClusterThreads * 8 * VPT;
  const T* gr = gu + static_cast<int64_t>(row) * 2 * I;
  float y[VPT][8];
  float amax = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = base + (v * kSiluClusterThreads + threadIdx.x) * 8;
    if (c < I) {
      float g[8], u[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(gr + c), g);
      unpack8<T>(*reinterpret_cast<const uint4*>(gr + I + c), u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        y[v][i] = Act<T>::to_float(Act<T>::from_float((g[i] / (1.0f + expf(-g[i]))) * u[i]));
        amax = fmaxf(amax, fabsf(y[v][i]));
      }
    }
  }
  const float local = block_max(amax, red);
  if (threadIdx.x < C) {  // thread r stores this CTA's maximum into CTA r's slot[rank]
    st_cluster_f32(mapa_shared(smem_u32(&slot[rank]), static_cast<uint32_t>(threadIdx.x)), local);
  }
  cluster_sync_all();
  float rmax = slot[0];
  for (int r = 1; r < C; ++r) rmax = fmaxf(rmax, slot[r]);
  const float sc = __fdiv_rn(rmax, 448.0f);
  if (rank == 0 && threadIdx.x == 0) qscale[row] = sc;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = base + (v * kSiluClusterThreads + threadIdx.x) * 8;
    if (c < I) *reinterpret_cast<uint2*>(qout + static_cast<int64_t>(row) * I + c) = e4m3x8(y[v], sc);
  }
}

// Rotate-half RoPE of one (first-half, second-half) pair with explicit
// roundings (no contraction into fma), so that every kernel that rotates —
// the RoPE + KV write kernels and the attention that fuses them — gives the
// same bits: (x0 c - x1 s, x1 c + x0 s).
__device__ __forceinline__ float2 rope_pair(float x0, float x1, float c, float s) {
  return make_float2(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)),
                     __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)));
}

// Vectorised RoPE + KV write for head sizes with 16-byte aligned half-rows
// (d % 16 == 0): CTA (sequence, item block); an item is 8 columns of the first
// half of one q / k head with the matching 8 of the second half (rotated), or
// 8 columns of one v head (copied).
template <typename T>
__global__ void __launch_bounds__(128) rope_kv_vec_kernel(
    T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache,
    const T* __restrict__ qkv, const T* __restrict__ cosv, const T* __restrict__ sinv,
    const int32_t* __restrict__ tables, const int32_t* __restrict__ positions, int hq, int hkv,
    int d, int block_size, int max_blocks) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int half = d / 2, oct = half / 8, dv = d / 8;
  const int rot = (hq + hkv) * oct;
  const int it = blockIdx.y * blockDim.x + threadIdx.x;
  if (it >= rot + hkv * dv) return;
  const T* row = qkv + static_cast<int64_t>(b) * (hq + 2 * hkv) * d;
  const int pos = positions[b];
  const bool in_cache = pos >= 0 && pos < max_blocks * block_size;
  const int blk = in_cache ? tables[static_cast<int64_t>(b) * max_blocks + pos / block_size] : 0;
  const int off = in_cache ? pos % block_size : 0;
  if (it < rot) {
    const int h = it / oct, c = (it - h * oct) * 8;
    float x0[8], x1[8], cs[8], sn[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(row + h * d + c), x0);
    unpack8<T>(*reinterpret_cast<const uint4*>(row + h * d + half + c), x1);
    unpack8<T>(*reinterpret_cast<const uint4*>(cosv + c), cs);
    unpack8<T>(*reinterpret_cast<const uint4*>(sinv + c), sn);
    uint4 p0, p1;
    T* r0 = reinterpret_cast<T*>(&p0);
    T* r1 = reinterpret_cast<T*>(&p1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 rr = rope_pair(x0[i], x1[i], cs[i], sn[i]);
      r0[i] = Act<T>::from_float(rr.x);  // rotate-half: first half
      r1[i] = Act<T>::from_float(rr.y);  // second half
    }
    T* dst;
    if (h < hq) {
      dst = q_out + (static_cast<int64_t>(b) * hq + h) * d;
    } else if (in_cache) {
      dst = k_cache + ((static_cast<int64_t>(blk) * hkv + (h - hq)) * block_size + off) * d;
    } else {
      return;
    }
    *reinterpret_cast<uint4*>(dst + c) = p0;
    *reinterpret_cast<uint4*>(dst + half + c) = p1;
  } else if (in_cache) {
    const int e = it - rot;
    const int kh = e / dv, c = (e - kh * dv) * 8;
    *reinterpret_cast<uint4*>(v_cache + ((static_cast<int64_t>(blk) * hkv + kh) * block_size + off) * d + c) =
        *reinterpret_cast<const uint4*>(row + (hq + hkv) * d + kh * d + c);
  }
}

// General head sizes (d even): one CTA per sequence, scalar accesses.
// qkv row: [q (hq*d) | k (hkv*d) | v (hkv*d)].
// cos/sin: d/2 entries for this step's position.  Cache: paged, block table row
// `tables[b]`, block_size positions per block.
template <typename T>
__global__ void __launch_bounds__(256) rope_kv_kernel(
    T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache,
    const T* __restrict__ qkv, const T* __restrict__ cosv, const T* __restrict__ sinv,
    const int32_t* __restrict__ tables, const int32_t* __restrict__ positions, int hq, int hkv,
    int d, int block_size, int max_blocks) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int half = d / 2;
  const T* row = qkv + static_cast<int64_t>(b) * (hq + 2 * hkv) * d;
  const int pos = positions[b];
  // a position outside the table's span writes q only (no cache access)
  const bool in_cache = pos >= 0 && pos < max_blocks * block_size;
  const int blk = in_cache ? tables[static_cast<int64_t>(b) * max_blocks + pos / block_size] : 0;
  const int off = in_cache ? pos % block_size : 0;
  const int pairs = (hq + hkv) * half;
  for (int e = threadIdx.x; e < pairs + hkv * d; e += blockDim.x) {
    if (e < pairs) {
      const int h = e / half, c = e - h * half;
      const T* src = row + h * d;
      const float x0 = Act<T>::to_float(src[c]), x1 = Act<T>::to_float(src[c + half]);
      const float cs = Act<T>::to_float(cosv[c]), sn = Act<T>::to_float(sinv[c]);
      const float2 rr = rope_pair(x0, x1, cs, sn);
      const T r0 = Act<T>::from_float(rr.x);   // rotate-half: first half
      const T r1 = Act<T>::from_float(rr.y);   // second half
      if (h < hq) {
        T* dst = q_out + (static_cast<int64_t>(b) * hq + h) * d;
        dst[c] = r0;
        dst[c + half] = r1;
      } else if (in_cache) {
        const int kh = h - hq;
        T* dst = k_cache + ((static_cast<int64_t>(blk) * hkv + kh) * block_size + off) * d;
        dst[c] = r0;
        dst[c + half] = r1;
      }
    } else if (in_cache) {
      const int e2 = e - pairs;
      const int kh = e2 / d, c = e2 - kh * d;
      v_cache[((static_cast<int64_t>(blk) * hkv + kh) * block_size + off) * d + c] =
          row[(hq + hkv) * d + kh * d + c];
    }
  }
}

// ------------------------------------------------------------ attention
constexpr int kAttnD = 128;        // head size
constexpr int kAttnTile = 64;      // positions per CTA iteration (16 per warp)
constexpr int kAttnThreads = 128;  // 4 warps
constexpr int kAttnRowBytes = kAttnD * 2 + 16;  // padded smem row (conflict-free ldmatrix)
constexpr int kAttnMaxBlocks = 512;  // block-table entries of one split cached in smem
constexpr int kAttnMaxCluster = 8;   // splits that merge in one cluster's shared memory
constexpr int kAttnMaxSplits = 256;  // splits that merge through the global workspace
constexpr int kAttnPartStride = 132; // split partial row: O[128], m, l, pad (16-byte rows)
// dynamic shared memory: per warp NS stages of 16 K + 16 V rows (at least the
// end-of-kernel warp merge buffer), then the split partial [16 rows][132]
__host__ __device__ constexpr int attn_main_smem(int ns) {
  return 4 * ns * 2 * 16 * kAttnRowBytes > 4 * 16 * (kAttnD + 2) * 4
             ? 4 * ns * 2 * 16 * kAttnRowBytes
             : 4 * 16 * (kAttnD + 2) * 4;
}
__host__ __device__ constexpr int attn_smem_bytes(int ns) {
  return attn_main_smem(ns) + 16 * kAttnPartStride * 4;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
struct MmaT;
template <>
struct MmaT<__half> {
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <>
struct MmaT<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// Merge n split partials (m, l in the log2 domain, unnormalised O over 16 dims)
// in source order into (M, L, acc), the loads of kB sources in flight at once:
// load(src, ml, o) fetches source src's (m, l) and its 16 O values.
template <int kB, typename Load>
__device__ __forceinline__ void attn_merge_sources(int n, Load load, float& M, float& L,
                                                   float (&acc)[16]) {
  M = -INFINITY;
  L = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  for (int s0 = 0; s0 < n; s0 += kB) {
    float2 ml[kB];
    float4 o[kB][4];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      if (s0 + j < n) {
        load(s0 + j, ml[j], o[j]);
      } else {
        ml[j] = make_float2(-INFINITY, 0.f);
#pragma unroll
        for (int q = 0; q < 4; ++q) o[j][q] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float bm = M;
#pragma unroll
    for (int j = 0; j < kB; ++j) bm = fmaxf(bm, ml[j].x);
    if (bm == -INFINITY) continue;          // every source so far is empty
    const float c = exp2f(M - bm);          // 0 while M is still -inf
    L *= c;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] *= c;
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const float f = exp2f(ml[j].x - bm);  // 0 for an empty source
      L += f * ml[j].y;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[4 * q] += f * o[j][q].x;
        acc[4 * q + 1] += f * o[j][q].y;
        acc[4 * q + 2] += f * o[j][q].z;
        acc[4 * q + 3] += f * o[j][q].w;
      }
    }
    M = bm;
  }
}

// grid: (num_seqs * num_kv_heads, splits).  Each CTA: one (sequence, KV head),
// positions [split * span, (split + 1) * span) of the context, the G q heads
// that read this KV head (G <= 16; rows >= G are padding).
// kv_map 0: q head h reads KV head h % num_kv_heads (the reference's paged
// kernel); 1: h / G (grouped, as torch's enable_gqa).
// splits == 1: writes out directly.  Otherwise the splits of one (sequence, KV
// head) form clusters of min(splits, kAttnMaxCluster) consecutive splits (grid y
// = splits, cluster y = that size; more than kAttnMaxCluster splits come in
// whole clusters).  Each CTA leaves its (O, m, l) partial in shared memory and,
// after a cluster barrier, the CTAs of a cluster share out the (row, 16-dim)
// items and merge their cluster's partials in split order through distributed
// shared memory.  One cluster writes the result.  Several (small batches: at
// batch 1 a CTA walking 512 positions alone took ~15 us whatever the KV size)
// write one merged partial per cluster into the global workspace (ws_part), and
// the last cluster of the (sequence, KV head) to arrive on its counter merges
// those in cluster order and sets the counter back to zero; no CTA waits on
// another cluster.  Both levels are deterministic.
// ROPE: RoPE and the KV-cache write of the new token fused in (what
// rope_kv_kernel does before the attention).  query is then the merged qkv row
// [seqs, (num_heads + 2 num_kv_heads) * 128]; each CTA rotates its q heads in
// registers (a lane holds both halves of each of its rotate-half pairs: k-steps
// kk and kk + 4); the warp whose tile holds the new token's position
// (context_lens - 1) rotates the token's k, lays k and v over that row of its
// tile in shared memory (the copy from the cache brought the old contents) and
// writes them into the cache after its loop.  Same bits as rope_kv_kernel
// followed by the plain attention (rope_pair in both).
template <typename T, int NS, bool ROPE>
__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(
    T* __restrict__ out, const T* __restrict__ query,
    const T* __restrict__ k_cache, const T* __restrict__ v_cache,
    const int32_t* __restrict__ tables, const int32_t* __restrict__ ctx_lens, int num_heads,
    int num_kv_heads, int block_size, int max_blocks, int span, float scale_log2, int kv_map,
    float* __restrict__ ws_part, uint32_t* __restrict__ ws_count, uint8_t* __restrict__ qout,
    float* __restrict__ qscale, const T* __restrict__ cosv, const T* __restrict__ sinv,
    T* __restrict__ kc_new, T* __restrict__ vc_new) {
  pdl_wait();
  pdl_trigger();
  // per warp [NS stages][K 16 rows | V 16 rows], rows padded to kAttnRowBytes;
  // then this split's partial (attn_smem_bytes)
  extern __shared__ __align__(16) uint8_t sm[];
  const int seq = blockIdx.x / num_kv_heads, kvh = blockIdx.x % num_kv_heads;
  const int split = blockIdx.y, splits = gridDim.y;
  const int G = num_heads / num_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  // never past the block table's span, never negative
  const int ctx = max(0, min(ctx_lens[seq], max_blocks * block_size));
  const int p0 = split * span;
  const int p1 = min(ctx, p0 + span);
  auto qhead = [&](int i) { return kv_map ? kvh * G + i : kvh + i * num_kv_heads; };

  // the split's block-table entries, read once into shared memory (the staging
  // loop would otherwise wait on a dependent global load before every copy)
  __shared__ int sblk[kAttnMaxBlocks];
  const int blk0 = p0 / block_size;
  const int nblk = p1 > p0 ? (p1 - 1) / block_size - blk0 + 1 : 0;
  const bool cached = nblk <= kAttnMaxBlocks;
  if (cached)
    for (int i = threadIdx.x; i < nblk; i += kAttnThreads)
      sblk[i] = tables[static_cast<int64_t>(seq) * max_blocks + blk0 + i];
  // the merged qkv row of this sequence (ROPE) / its q rows
  const int64_t qrow = ROPE ? static_cast<int64_t>(seq) * (num_heads + 2 * num_kv_heads) * kAttnD
                            : static_cast<int64_t>(seq) * num_heads * kAttnD;
  // ROPE: the warp whose tile holds the new token's position (context_lens - 1,
  // inside this split) requests the token's k pairs (c, c + 64) for c = lane,
  // lane + 32, the matching cos / sin and v columns 4 lane .. + 3; it patches
  // the rotated row into that tile in shared memory once the tile's copies have
  // landed, and writes it into the cache after the loop, so that no other work
  // of the CTA waits for it
  int rope_tile = -1, rope_row = 0;  // the warp's tile index holding the token, its row
  T rk[4], rc[2], rs[2];
  uint2 rv = make_uint2(0u, 0u);
  int64_t rope_off = 0;
  if constexpr (ROPE) {
    const int pos = ctx_lens[seq] - 1;
    const int ti = (pos - p0) >> 4;
    if (pos >= p0 && pos < p1 && (ti & 3) == warp) {
      rope_tile = ti >> 2;
      rope_row = (pos - p0) & 15;
      const T* kr = query + qrow + static_cast<int64_t>(num_heads + kvh) * kAttnD;
      const T* vr = query + qrow + static_cast<int64_t>(num_heads + num_kv_heads + kvh) * kAttnD;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = lane + 32 * h;
        rk[2 * h] = kr[c];
        rk[2 * h + 1] = kr[c + kAttnD / 2];
        rc[h] = cosv[c];
        rs[h] = sinv[c];
      }
      rv = *reinterpret_cast<const uint2*>(vr + 4 * lane);
      const int blk = tables[static_cast<int64_t>(seq) * max_blocks + pos / block_size];
      rope_off =
          ((static_cast<int64_t>(blk) * num_kv_heads + kvh) * block_size + pos % block_size) * kAttnD;
    }
  }
  __syncthreads();  // table entries in place

  // Q fragments (A operand, 16 rows = q heads, 128 dims = 8 k-steps)
  uint32_t qa[8][4];
  {
    const bool r0 = g < G, r1 = g + 8 < G;
    const T* q0 = query + qrow + static_cast<int64_t>(r0 ? qhead(g) : 0) * kAttnD;
    const T* q1 = query + qrow + static_cast<int64_t>(r1 ? qhead(g + 8) : 0) * kAttnD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 16 + 2 * t;
      qa[kk][0] = r0 ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
      qa[kk][1] = r1 ? *reinterpret_cast<const uint32_t*>(q1 + c) : 0u;
      qa[kk][2] = r0 ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
      qa[kk][3] = r1 ? *reinterpret_cast<const uint32_t*>(q1 + c + 8) : 0u;
    }
    if constexpr (ROPE) {
      // register i of k-step kk holds columns c, c + 1 (c = 16 kk + 2t, + 8 for
      // i >= 2); for kk < 4 its rotate-half partners sit in k-step kk + 4
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = kk * 16 + 2 * t + ((i & 2) ? 8 : 0);
          const float2 cs = unpack2<T>(*reinterpret_cast<const uint32_t*>(cosv + c));
          const float2 sn = unpack2<T>(*reinterpret_cast<const uint32_t*>(sinv + c));
          const float2 a = unpack2<T>(qa[kk][i]), b = unpack2<T>(qa[kk + 4][i]);
          const float2 e0 = rope_pair(a.x, b.x, cs.x, sn.x), e1 = rope_pair(a.y, b.y, cs.y, sn.y);
          qa[kk][i] = pack2<T>(e0.x, e1.x);
          qa[kk + 4][i] = pack2<T>(e0.y, e1.y);
        }
      }
    }
  }

  // Each warp streams its own 16-position tiles (tiles warp, warp + 4, ... of the
  // split) through an NS-stage cp.async ring in its own shared-memory region: no
  // CTA-wide barrier inside the loop.
  constexpr int kWarpTile = 16 * kAttnRowBytes;          // K (or V) rows of one tile
  constexpr int kWarpStage = 2 * kWarpTile;
  uint8_t* wsm = sm + warp * NS * kWarpStage;
  auto stage = [&](int j, int buf) {
    const uint32_t kb = smem_u32(wsm + buf * kWarpStage);
    const uint32_t vb = kb + kWarpTile;
    const int base = p0 + (warp + 4 * j) * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 2 * i + (lane >> 4), ch = lane & 15;
      const int pos = base + r;
      const bool ok = pos < p1;
      const int pp = ok ? pos : p0;
      const int bi = pp / block_size;
      const int blk = cached ? sblk[bi - blk0] : tables[static_cast<int64_t>(seq) * max_blocks + bi];
      const int64_t off = ((static_cast<int64_t>(blk) * num_kv_heads + kvh) * block_size +
                           pp % block_size) * kAttnD + ch * 8;
      cp_async16(kb + r * kAttnRowBytes + ch * 16, k_cache + off, ok);
      cp_async16(vb + r * kAttnRowBytes + ch * 16, v_cache + off, ok);
    }
    cp_async_commit();
  };

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g, g+8

  const int ntiles_all = p1 > p0 ? (p1 - p0 + 15) / 16 : 0;
  const int ntiles = ntiles_all > warp ? (ntiles_all - warp + 3) / 4 : 0;  // this warp's
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) {
    if (i < ntiles) stage(i, i);
    else cp_async_commit();  // empty group keeps the group count uniform
  }
  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile % NS;
    cp_async_wait<NS - 2>();  // this tile's group has landed for this lane ...
    __syncwarp();             // ... and for every lane; tile - 1's buffer is free
    if constexpr (ROPE) {
      if (tile == rope_tile) {  // the new token's row: rotated k and v over the copied row
        T* krow = reinterpret_cast<T*>(wsm + buf * kWarpStage + rope_row * kAttnRowBytes);
        T* vrow = reinterpret_cast<T*>(wsm + buf * kWarpStage + kWarpTile + rope_row * kAttnRowBytes);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = lane + 32 * h;
          const float2 rr = rope_pair(Act<T>::to_float(rk[2 * h]), Act<T>::to_float(rk[2 * h + 1]),
                                      Act<T>::to_float(rc[h]), Act<T>::to_float(rs[h]));
          rk[2 * h] = Act<T>::from_float(rr.x);
          rk[2 * h + 1] = Act<T>::from_float(rr.y);
          krow[c] = rk[2 * h];
          krow[c + kAttnD / 2] = rk[2 * h + 1];
        }
        *reinterpret_cast<uint2*>(vrow + 4 * lane) = rv;
        __syncwarp();
      }
    }
    if (tile + NS - 1 < ntiles) stage(tile + NS - 1, (tile + NS - 1) % NS);
    else cp_async_commit();
    const uint32_t kb = smem_u32(wsm + buf * kWarpStage);
    const uint32_t vb = kb + kWarpTile;
    // S[16 heads x 16 positions] = Q K^T: B operand (k = dim, n = position) from K
    // rows (position-major) with ldmatrix (no transpose); two 8-position halves
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      // matrices: (pos 0-7, dims kk*16..+7), (pos 0-7, +8..15), (pos 8-15, dims ..), ...
      uint32_t kf[4];
      const int mi = lane >> 3, ri = lane & 7;
      // x4: m0 = pos 0-7 dims [16kk, +8), m1 = pos 0-7 dims [16kk+8, +8),
      //     m2 = pos 0-7 dims [16(kk+1), +8), m3 = pos 0-7 dims [16(kk+1)+8, +8)
      ldsm_x4(kf, kb + ri * kAttnRowBytes + (kk * 16 + mi * 8) * 2);
      MmaT<T>::mma(s[0], qa[kk], kf[0], kf[1]);
      MmaT<T>::mma(s[0], qa[kk + 1], kf[2], kf[3]);
      ldsm_x4(kf, kb + (8 + ri) * kAttnRowBytes + (kk * 16 + mi * 8) * 2);
      MmaT<T>::mma(s[1], qa[kk], kf[0], kf[1]);
      MmaT<T>::mma(s[1], qa[kk + 1], kf[2], kf[3]);
    }
    // mask, scale (log2 domain), online softmax for rows g (s[.][0..1]) and g+8 (s[.][2..3])
    const int pbase = p0 + (warp + 4 * tile) * 16;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const bool ok = pbase + h2 * 8 + 2 * t + j < p1;
        s[h2][j] = ok ? s[h2][j] * scale_log2 : -INFINITY;
        s[h2][2 + j] = ok ? s[h2][2 + j] * scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[h2][j]);
        mx1 = fmaxf(mx1, s[h2][2 + j]);
      }
#pragma unroll
    for (int o_ = 1; o_ < 4; o_ <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
    }
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float c0 = nm0 == -INFINITY ? 1.f : exp2f(m0 - nm0);
    const float c1 = nm1 == -INFINITY ? 1.f : exp2f(m1 - nm1);
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        s[h2][j] = nm0 == -INFINITY ? 0.f : exp2f(s[h2][j] - nm0);
        s[h2][2 + j] = nm1 == -INFINITY ? 0.f : exp2f(s[h2][2 + j] - nm1);
        ps0 += s[h2][j];
        ps1 += s[h2][2 + j];
      }
    l0 = l0 * c0 + ps0;  // per-lane partial row sums; reduced over t at the end
    l1 = l1 * c1 + ps1;
    m0 = nm0;
    m1 = nm1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= c0;
      o[n][1] *= c0;
      o[n][2] *= c1;
      o[n][3] *= c1;
    }
    // P (A operand, k = 16 positions) from the S accumulators
    uint32_t pa[4];
    pa[0] = MmaT<T>::pack(s[0][0], s[0][1]);
    pa[1] = MmaT<T>::pack(s[0][2], s[0][3]);
    pa[2] = MmaT<T>::pack(s[1][0], s[1][1]);
    pa[3] = MmaT<T>::pack(s[1][2], s[1][3]);
    // O += P V: B operand (k = position, n = dim) from V rows with ldmatrix.trans
#pragma unroll
    for (int n = 0; n < 16; n += 2) {
      uint32_t vf[4];
      const int mi = lane >> 3, ri = lane & 7;
      // x4.trans: m0 = pos 0-7 dims [8n, +8), m1 = pos 8-15 dims [8n, +8),
      //           m2 = pos 0-7 dims [8(n+1), +8), m3 = pos 8-15 dims [8(n+1), +8)
      ldsm_x4_t(vf, vb + ((mi & 1) * 8 + ri) * kAttnRowBytes + (n * 8 + (mi >> 1) * 8) * 2);
      MmaT<T>::mma(o[n], pa, vf[0], vf[1]);
      MmaT<T>::mma(o[n + 1], pa, vf[2], vf[3]);
    }
  }
  cp_async_wait<0>();
  if constexpr (ROPE) {
    if (rope_tile >= 0) {  // the new token into the cache (no copy of this CTA reads it now)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        kc_new[rope_off + lane + 32 * h] = rk[2 * h];
        kc_new[rope_off + lane + 32 * h + kAttnD / 2] = rk[2 * h + 1];
      }
      *reinterpret_cast<uint2*>(vc_new + rope_off + 4 * lane) = rv;
    }
  }

  // ---- merge the 4 warps (each covered a quarter of every tile)
#pragma unroll
  for (int o_ = 1; o_ < 4; o_ <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
  }
  float* mrg = reinterpret_cast<float*>(sm);  // [4 warps][16 rows][130] (O 128, m, l)
  constexpr int kStride = kAttnD + 2;
  float* part = reinterpret_cast<float*>(sm + attn_main_smem(NS));  // this split's partial
  __syncthreads();
  {
    float* wp = mrg + warp * 16 * kStride;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      wp[g * kStride + n * 8 + 2 * t] = o[n][0];
      wp[g * kStride + n * 8 + 2 * t + 1] = o[n][1];
      wp[(g + 8) * kStride + n * 8 + 2 * t] = o[n][2];
      wp[(g + 8) * kStride + n * 8 + 2 * t + 1] = o[n][3];
    }
    if (t == 0) {
      wp[g * kStride + kAttnD] = m0;
      wp[g * kStride + kAttnD + 1] = l0;
      wp[(g + 8) * kStride + kAttnD] = m1;
      wp[(g + 8) * kStride + kAttnD + 1] = l1;
    }
  }
  __syncthreads();
  // FP8 output (one KV head: a (sequence, KV head) is a whole token row): every
  // path below leaves at most one (row, 16-dim) item of the final output with a
  // thread, kept rounded in qv; the row's maximum, scale and e4m3 bytes then
  // follow fp8_quant_rows_kernel's arithmetic
  static_assert(16 * 8 <= kAttnThreads, "one output item per thread");
  __shared__ float qred[32];
  __shared__ float qslot[kAttnMaxCluster];
  float qv[16];
  int qe = -1;
  auto item_out = [&](int e, int r, int d0, const float (&acc)[16], float L) {
    T* dst = out + (static_cast<int64_t>(seq) * num_heads + qhead(r)) * kAttnD + d0;
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const T o = Act<T>::from_float(acc[i] * inv);
      dst[i] = o;
      qv[i] = Act<T>::to_float(o);
    }
    qe = e;
  };
  auto item_max = [&]() {
    float m = 0.f;
    if (qe >= 0) {
#pragma unroll
      for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(qv[i]));
    }
    return m;
  };
  auto item_e4m3 = [&](float rmax) {
    const float sc = __fdiv_rn(rmax, 448.0f);
    if (qe >= 0) {
      const int r = qe >> 3, d0 = (qe & 7) * 16;
      uint8_t* qd = qout + (static_cast<int64_t>(seq) * num_heads + qhead(r)) * kAttnD + d0;
      float lo[8], hi[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        lo[i] = qv[i];
        hi[i] = qv[8 + i];
      }
      *reinterpret_cast<uint2*>(qd) = e4m3x8(lo, sc);
      *reinterpret_cast<uint2*>(qd + 8) = e4m3x8(hi, sc);
    }
    return sc;
  };
  // thread -> (row r, 16 consecutive dims)
  for (int e = threadIdx.x; e < G * 8; e += kAttnThreads) {
    const int r = e >> 3, d0 = (e & 7) * 16;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mrg[(w * 16 + r) * kStride + kAttnD]);
    float L = 0.f, acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* wr = mrg + (w * 16 + r) * kStride;
      const float f = M == -INFINITY ? 0.f : exp2f(wr[kAttnD] - M);
      L += f * wr[kAttnD + 1];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] += f * wr[d0 + i];
    }
    if (splits == 1) {
      item_out(e, r, d0, acc, L);
    } else {
      // partial: O (unnormalised, fp32), then m, l, in shared memory
      float* pw = part + r * kAttnPartStride;
#pragma unroll
      for (int i = 0; i < 16; ++i) pw[d0 + i] = acc[i];
      if (d0 == 0) {
        pw[kAttnD] = M;
        pw[kAttnD + 1] = L;
      }
    }
  }
  if (splits == 1) {
    if (qout != nullptr) {
      const float sc = item_e4m3(block_max(item_max(), qred));
      if (threadIdx.x == 0) qscale[seq] = sc;
    }
    return;
  }
  // ---- first level: the cluster's splits, through distributed shared memory
  const int cs = splits < kAttnMaxCluster ? splits : kAttnMaxCluster;  // cluster size
  const int crank = split % cs, nclu = splits / cs, clu = split / cs;
  cluster_sync_all();   // every split's partial is in its CTA's shared memory
  const uint32_t part_u32 = smem_u32(part);
  for (int e = threadIdx.x * cs + crank; e < G * 8; e += kAttnThreads * cs) {
    const int r = e >> 3, d0 = (e & 7) * 16;
    const uint32_t row = part_u32 + static_cast<uint32_t>(r * kAttnPartStride) * 4u;
    float M, L, acc[16];
    attn_merge_sources<4>(cs, [&](int src, float2& ml, float4 (&o)[4]) {
      const uint32_t pr = mapa_shared(row, static_cast<uint32_t>(src));
      const float4 m4 = ld_cluster_v4(pr + kAttnD * 4u);
      ml = make_float2(m4.x, m4.y);
#pragma unroll
      for (int q = 0; q < 4; ++q) o[q] = ld_cluster_v4(pr + static_cast<uint32_t>(d0 + 4 * q) * 4u);
    }, M, L, acc);
    if (nclu == 1) {
      item_out(e, r, d0, acc, L);
    } else {   // this cluster's partial, item by item, into the workspace
      float* pw = ws_part + ((static_cast<int64_t>(blockIdx.x) * nclu + clu) * 16 + r) * kAttnPartStride;
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        __stcg(reinterpret_cast<float4*>(pw + d0 + i), make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
      if (d0 == 0) __stcg(reinterpret_cast<float2*>(pw + kAttnD), make_float2(M, L));
    }
  }
  // FP8, one cluster: each CTA's maximum into slot[rank] of every CTA
  if (qout != nullptr && nclu == 1) {
    const float m = block_max(item_max(), qred);
    if (threadIdx.x < cs)
      st_cluster_f32(mapa_shared(smem_u32(&qslot[crank]), static_cast<uint32_t>(threadIdx.x)), m);
  }
  // no CTA leaves while a peer may read its partial; the release / acquire of
  // the cluster barrier also orders every thread's workspace items before the
  // arrival below (the CTA-barrier-then-one-fenced-atomic pattern)
  cluster_sync_all();
  if (nclu == 1) {
    if (qout != nullptr) {
      float rmax = qslot[0];
      for (int q = 1; q < cs; ++q) rmax = fmaxf(rmax, qslot[q]);
      const float sc = item_e4m3(rmax);
      if (crank == 0 && threadIdx.x == 0) qscale[seq] = sc;
    }
    return;
  }
  // ---- second level: the cluster partials, by the last cluster to arrive
  __shared__ uint32_t s_last;
  if (threadIdx.x == 0) {
    bool last = false;
    if (crank == 0) {
      __threadfence();   // the cluster's partial, before its arrival
      last = atomicAdd(ws_count + blockIdx.x, 1u) == static_cast<uint32_t>(nclu - 1);
      if (last) __threadfence();   // every cluster's partial, after the last arrival
    }
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  const float* pbase = ws_part + static_cast<int64_t>(blockIdx.x) * nclu * 16 * kAttnPartStride;
  for (int e = threadIdx.x; e < G * 8; e += kAttnThreads) {
    const int r = e >> 3, d0 = (e & 7) * 16;
    float M, L, acc[16];
    attn_merge_sources<8>(nclu, [&](int src, float2& ml, float4 (&o)[4]) {
      const float* pr = pbase + (src * 16 + r) * kAttnPartStride;
      ml = __ldcg(reinterpret_cast<const float2*>(pr + kAttnD));
#pragma unroll
      for (int q = 0; q < 4; ++q) o[q] = __ldcg(reinterpret_cast<const float4*>(pr + d0 + 4 * q));
    }, M, L, acc);
    item_out(e, r, d0, acc, L);
  }
  if (qout != nullptr) {
    const float sc = item_e4m3(block_max(item_max(), qred));
    if (threadIdx.x == 0) qscale[seq] = sc;
  }
  if (threadIdx.x == 0) ws_count[blockIdx.x] = 0u;  // ready for the next call
}

}  // namespace lmrs
