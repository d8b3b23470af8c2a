// awq_i8.cuh — AWQ W4A16 decode GEMV for 1-2 tokens on the integer tensor path.
//
// y[m, n] = sum_g s[g, n] * sum_{k in g} (q[k, n] - z[g, n]) * x[m, k]
//
// The register-fed GEMVs (awq_gemv*.cuh) turn every nibble into an fp16 MMA
// operand with integer lop3/prmt work that costs about as much as streaming the
// weights, so unpacking and streaming run back to back.  This kernel does no
// per-weight unpacking at all: the packed bytes ARE the MMA operand.
//   * A byte of an AWQ word holds two columns: lo + 16 * hi.  One
//     mma.m16n8k32.u8.s8 on the raw bytes gives R = L + 16 H per byte column
//     (L, H the dot products of the low / high nibbles); a second on the bytes
//     masked with 0xF0 (one lop3 per four bytes) gives 16 H.  Both are exact
//     integers.
//   * The activations become integers without loss that matters: per box of
//     BR rows and per token, X = rint(x * 2^sh) with sh chosen so |X| < 2^22
//     (every fp16 value within 2^11 of the box maximum is exact, every bf16
//     one within 2^14; the rest are rounded at 2^-22 of the maximum, below
//     fp32 accumulation noise), split
//     into three balanced signed bytes X = d0 + 256 d1 + 65536 d2.  Each limb
//     is one MMA column, so a box's integer sums are exact.
//   * No byte transposes: the K slots of an A register are the four bytes of
//     one packed word (four byte columns of one row), and the B fragment is
//     "diagonal": MMA column n = 2 i + slot carries its limb only in byte i, so
//     D[word][n] sums byte i of that word over the step's eight rows.  Lane
//     (g, t) ends up holding byte t of words 2g and 2g+1 of each 16-word tile,
//     all three limbs of each token, so the fix-up needs no shuffles.
//   * Zero point and scale once per box: y += s * 2^-sh * ((R - 16H) - z SX,
//     16H - 16 z SX) with SX = sum of the box's limbs, exact in integers.
// Pipeline: one producer thread streams boxes (BR rows x 32 packed words, 128-
// byte swizzle), the group's scale and zero rows and the box's rows of x into a
// ring with TMA (one lane per slot for the first pass), the weights of the first
// slots before griddepcontrol.wait; a converter warp turns each box's x into
// limbs inside the slot; four consumer warps (one per SM sub-partition) take
// the two 16-word tiles of alternate boxes.
// A cluster of C CTAs splits one 256-column strip's K; partial sums meet in
// the owner CTA's shared memory through st.async (as in awq_gemv4.cuh).
#pragma once
#include <cooperative_groups.h>
#include "awq_gemv.cuh"
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kI8Words = 32;             // packed words per strip row
constexpr int kI8Strip = 8 * kI8Words;   // 256 output columns
constexpr int kI8Streams = 2;            // box streams (alternate boxes)
constexpr int kI8Consumers = 2 * kI8Streams;    // consumer warps: stream x 16-word tile
constexpr int kI8Producer = kI8Consumers;       // TMA issue
constexpr int kI8Converter = kI8Consumers + 1;  // x -> limbs, box by box
constexpr int kI8Threads = 32 * (kI8Consumers + 2);
constexpr int kI8MaxCluster = 8;

// Ring slot s: the packed box at box(s) (1024-byte aligned for the 128-byte
// swizzle) and, in a second ring, scale row | zero row | x rows (fp16,
// [token][row]) | limbs | per-token (2^-sh, SX0, SX1, SX2) at ext(s), each part
// 128-byte aligned.
template <int TOK, int BR>
struct AwqI8Layout {
  static constexpr int kBox = BR * kI8Words * 4;   // packed words of one box
  static constexpr int kScale = kI8Strip * 2;      // fp16 scale row
  static constexpr int kZero = kI8Words * 4;       // packed zero row
  static constexpr int kX = BR * 2 * TOK;          // the box's rows of x
  static constexpr int kXRow = 4 * TOK;            // limb bytes per row: (d0, d1, d2, 0) per token
  static constexpr int kOffScale = 0;
  static constexpr int kOffZero = kOffScale + kScale;
  static constexpr int kOffX = kOffZero + kZero;
  static constexpr int kOffLimb = kOffX + (kX + 127) / 128 * 128;
  static constexpr int kOffInfo = kOffLimb + (BR * kXRow + 127) / 128 * 128;
  static constexpr int kExtra = (kOffInfo + 16 * TOK + 127) / 128 * 128;
  static constexpr int kTxW = kBox + kScale + kZero;  // issued before griddepcontrol.wait
  static constexpr int kTx = kTxW + kX;
  static constexpr int kVar = (3 * TOK + 1) / 2;   // MMA column sets: 2 limbs each
  static constexpr int kRecvCols = kI8Strip + kI8MaxCluster;
  static constexpr int kRecv = kRecvCols * 16;     // [source rank][owner column] float4
  static constexpr int kRed = kI8Streams * TOK * kI8Strip * 4;
  static_assert(BR == 64 || BR == 128, "box rows");
  static_assert(TOK == 1 || TOK == 2, "tokens");
  static_assert(kRed <= kBox, "the drained ring holds the partials");
  __host__ __device__ static constexpr int smem_bytes(int S) {
    return 1024 + S * (kBox + kExtra) + kRecv + (3 * S + 1) * 8;
  }
};

__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Owner split of a strip's 256 columns over C cluster ranks (uneven for C not
// a power of two).
__device__ __forceinline__ int i8_col_lo(int r, int C) { return (r * kI8Strip) / C; }

template <int TOK, int BR, typename T>
__global__ void __launch_bounds__(kI8Threads, 1) awq_gemv_i8_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_s,
    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_x,
    T* __restrict__ y, const T* __restrict__ bias, int M, int K, int N, int group,
    int S) {
  using L = AwqI8Layout<TOK, BR>;
  constexpr int V = L::kVar;
  constexpr int RPL = BR / 32;  // x rows per lane in the limb conversion
  extern __shared__ uint8_t smem_raw[];
  // offset from the shared array itself, so every access below stays a
  // shared-memory access
  uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int nb_all = K / BR;
  const int b_lo = static_cast<int>((static_cast<long long>(rank) * nb_all) / C);
  const int b_hi = static_cast<int>((static_cast<long long>(rank + 1) * nb_all) / C);
  const int nbox = b_hi - b_lo;

  uint8_t* extra = ring + S * L::kBox;
  auto box = [&](int s) { return ring + s * L::kBox; };
  auto ext = [&](int s) { return extra + s * L::kExtra; };
  float4* recv = reinterpret_cast<float4*>(extra + S * L::kExtra);
  uint64_t* full = reinterpret_cast<uint64_t*>(recv + L::kRecvCols);
  uint64_t* xready = full + S;
  uint64_t* empty = xready + S;
  uint64_t* recv_bar = empty + S;

  const int my_lo = i8_col_lo(rank, C), my_cols = i8_col_lo(rank + 1, C) - my_lo;
  const int cwmax = (kI8Strip + C - 1) / C;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&xready[i], 1);
      mbar_init(&empty[i], 2);  // the box's two tile warps
    }
    // the owner's own arrive plus C x my_cols 16-byte st.async deliveries
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(C * my_cols * 16));
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive_relaxed();
  pdl_trigger();

  const int g = lane >> 2, t = lane & 3;
  float acc[2][TOK][2];   // [word 2g / 2g+1 of the tile][token][lo / hi column]
#pragma unroll
  for (int w = 0; w < 2; ++w)
#pragma unroll
    for (int m = 0; m < TOK; ++m) acc[w][m][0] = acc[w][m][1] = 0.f;

  if (warp == kI8Producer) {
    // ---------------- producer: weights of the first slots before the wait on
    // the previous kernel, x rows after it, then refill the ring
    const int pre = nbox < S ? nbox : S;
    if (lane == 0) tma_prefetch_desc(&tm_q);
    if (lane == 1) tma_prefetch_desc(&tm_s);
    if (lane == 2) tma_prefetch_desc(&tm_z);
    if (lane == 3) tma_prefetch_desc(&tm_x);
    if (lane < pre) {   // lane b issues box b of the first ring pass
      const int c0 = strip * kI8Words;
      auto load_weights = [&](int b, int s) {
        const int krow = (b_lo + b) * BR;
        const int gi = krow / group;
        mbar_arrive_expect_tx(&full[s], L::kTx);
        tma_load_2d(&tm_q, &full[s], box(s), c0, krow);
        tma_load_2d(&tm_s, &full[s], ext(s) + L::kOffScale, strip * kI8Strip, gi);
        tma_load_2d(&tm_z, &full[s], ext(s) + L::kOffZero, c0, gi);
      };
      auto load_x = [&](int b, int s) {
        tma_load_2d(&tm_x, &full[s], ext(s) + L::kOffX, (b_lo + b) * BR, 0);
      };
      load_weights(lane, lane);
      pdl_wait();
      load_x(lane, lane);
      int s = 0;
      uint32_t ph = 0;
      for (int b = lane == 0 ? pre : nbox; b < nbox; ++b) {
        if (!mbar_wait(&empty[s], ph, kErrWaitEmpty)) break;
        load_weights(b, s);
        load_x(b, s);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == kI8Converter) {
    // ---------------- converter: per box and token, X = rint(x 2^sh) with
    // |X| < 2^22, split into balanced signed bytes d0 + 256 d1 + 65536 d2
    int s = 0;
    uint32_t ph = 0;
    for (int b = 0; b < nbox; ++b) {
      if (!mbar_wait(&full[s], ph, kErrWaitFull)) break;
      uint8_t* slot = ext(s);
#pragma unroll
      for (int tok = 0; tok < TOK; ++tok) {
        const uint8_t* xp = slot + L::kOffX + (tok * BR + lane * RPL) * 2;
        float v[RPL];
        if constexpr (RPL == 4) {
          const uint2 raw = ld_s64(xp);
          const float2 f0 = Act<T>::unpack2(raw.x), f1 = Act<T>::unpack2(raw.y);
          v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
        } else {
          const float2 f0 = Act<T>::unpack2(ld_s32(xp));
          v[0] = f0.x; v[1] = f0.y;
        }
        float m = 0.f;
        bool bad = false;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const float a = fabsf(v[i]);
          bad |= !(a <= Act<T>::kMaxFinite);   // NaN or Inf
          m = fmaxf(m, a);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad = __any_sync(0xffffffffu, bad);
        // |X| < 2^(e+1) * 2^(21-e) = 2^22.  fp16 values are normal fp32 numbers
        // (sh <= 45); bf16 ones span the fp32 range, so sh is capped at 126 to
        // keep 2^sh and 2^-sh normal (a box whose maximum is below 2^-105 then
        // keeps fewer than 22 bits: values that small vanish in fp32 sums anyway)
        const int e = m > 0.f ? ((__float_as_int(m) >> 23) & 255) - 127 : 0;
        const int sh = m > 0.f ? min(21 - e, 126) : 0;
        const float scl = __int_as_float((sh + 127) << 23);
        int sx0 = 0, sx1 = 0, sx2 = 0;
        uint8_t* xr = slot + L::kOffLimb + lane * RPL * L::kXRow + 4 * tok;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int X = bad ? 0 : __float2int_rn(v[i] * scl);
          const int d0 = ((X + 128) & 255) - 128;
          const int X1 = (X - d0) >> 8;
          const int d1 = ((X1 + 128) & 255) - 128;
          const int d2 = (X1 - d1) >> 8;
          sx0 += d0; sx1 += d1; sx2 += d2;
          *reinterpret_cast<uint32_t*>(xr + i * L::kXRow) =
              static_cast<uint32_t>(d0 & 255) | (static_cast<uint32_t>(d1 & 255) << 8) |
              (static_cast<uint32_t>(d2 & 255) << 16);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          sx0 += __shfl_xor_sync(0xffffffffu, sx0, o);
          sx1 += __shfl_xor_sync(0xffffffffu, sx1, o);
          sx2 += __shfl_xor_sync(0xffffffffu, sx2, o);
        }
        if (lane == 0) {
          const float p = bad ? __int_as_float(0x7fc00000) : __int_as_float((127 - sh) << 23);
          *reinterpret_cast<int4*>(slot + L::kOffInfo + 16 * tok) =
              make_int4(__float_as_int(p), sx0, sx1, sx2);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&xready[s]);
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
    }
  } else {
    // ---------------- consumers: warp (p, tl) takes the 16-word tile tl of boxes
    // p, p+2, ...
    const int p = warp >> 1, tl = warp & 1;
    // Rows of the 8-row step: a0/a1 and b0 use row rho, a2/a3 and b1 row rho + 2;
    // rho = 0,1,4,5 for t = 0..3 keeps each 64-bit LDS at two addresses per bank
    // under the 128-byte swizzle (chunk ^= row).
    const int rho = (t & 1) | ((t & 2) << 1);
    uint32_t offA[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = rho + 2 * h;
      offA[h] = static_cast<uint32_t>(r * 128 + ((((4 * tl + (g >> 1)) ^ r) & 7) << 4) +
                                      8 * (g & 1));
    }
    // B selectors: column n = g carries entry e = 2v + (g & 1) (token e / 3, limb
    // e % 3) in byte g >> 1, zero elsewhere
    uint32_t sel[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int e = 2 * v + (g & 1);
      const uint32_t sh4 = 4u * static_cast<uint32_t>(g >> 1);
      sel[v] = e < 3 * TOK ? ((0x4444u & ~(0xFu << sh4)) | (static_cast<uint32_t>(e % 3) << sh4))
                           : 0x4444u;
    }
    const bool odd = (g & 1) != 0;
    // this lane's columns: byte t of word w holds columns 8w + ORDER[2t], 8w + ORDER[2t+1]
    const int clo = (t >> 1) | ((t & 1) << 2);
    const int w0 = 16 * tl + 2 * g;   // this lane's words w0, w0 + 1
    int s = p;
    uint32_t ph = 0;
    for (int b = p; b < nbox; b += kI8Streams) {
      if (!mbar_wait(&full[s], ph, kErrWaitFull)) break;
      if (!mbar_wait(&xready[s], ph, kErrWaitDequant)) break;
      const uint8_t* wb = box(s);
      const uint8_t* eb = ext(s);
      // scales, zero words and the box's x figures, read before the slot is released
      const __half* sc = reinterpret_cast<const __half*>(eb + L::kOffScale);
      int4 xi[TOK];
#pragma unroll
      for (int m = 0; m < TOK; ++m) xi[m] = *reinterpret_cast<const int4*>(eb + L::kOffInfo + 16 * m);
      const uint2 z2 = ld_s64(eb + L::kOffZero + w0 * 4);
      const uint32_t zv[2] = {z2.x, z2.y};
      float sv[2][2];
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const int col = 8 * (w0 + w) + clo;
        sv[w][0] = __half2float(sc[col]);
        sv[w][1] = __half2float(sc[col + 2]);
      }
      int Dr[V][4], Dm[V][4];
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int c = 0; c < 4; ++c) Dr[v][c] = Dm[v][c] = 0;
      const uint8_t* xb = eb + L::kOffLimb;
#pragma unroll 4
      for (int st = 0; st < BR / 8; ++st) {
        const uint8_t* ws = wb + st * 1024;
        const uint8_t* xs = xb + st * 8 * L::kXRow;
        uint32_t xw0[TOK], xw1[TOK];
#pragma unroll
        for (int m = 0; m < TOK; ++m) {
          xw0[m] = ld_s32(xs + rho * L::kXRow + 4 * m);
          xw1[m] = ld_s32(xs + (rho + 2) * L::kXRow + 4 * m);
        }
        const uint2 p0 = ld_s64(ws + offA[0]);
        const uint2 p1 = ld_s64(ws + offA[1]);
        const uint32_t a[4] = {p0.x, p0.y, p1.x, p1.y};
        const uint32_t am[4] = {p0.x & 0xF0F0F0F0u, p0.y & 0xF0F0F0F0u, p1.x & 0xF0F0F0F0u,
                                p1.y & 0xF0F0F0F0u};
#pragma unroll
        for (int v = 0; v < V; ++v) {
          constexpr int kLast = TOK - 1;
          const int te = (2 * v) / 3 < kLast ? (2 * v) / 3 : kLast;
          const int to = (2 * v + 1) / 3 < kLast ? (2 * v + 1) / 3 : kLast;
          const uint32_t b0 = prmt(odd ? xw0[to] : xw0[te], 0u, sel[v]);
          const uint32_t b1 = prmt(odd ? xw1[to] : xw1[te], 0u, sel[v]);
          mma_u8s8_16832(Dr[v], a, b0, b1);
          mma_u8s8_16832(Dm[v], am, b0, b1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      // fix-up: entry e = 3 tok + j sits in Dx[e >> 1][2 w + (e & 1)]
#pragma unroll
      for (int m = 0; m < TOK; ++m) {
        const float pm = __int_as_float(xi[m].x);
        const int sxj[3] = {xi[m].y, xi[m].z, xi[m].w};
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int zlo = static_cast<int>((zv[w] >> (8 * t)) & 0xFu);
          const int zhi = static_cast<int>((zv[w] >> (8 * t + 4)) & 0xFu);
          float flo[3], fhi[3];
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const int e = 3 * m + j;
            const int R = Dr[e >> 1][2 * w + (e & 1)];
            const int H = Dm[e >> 1][2 * w + (e & 1)];
            flo[j] = static_cast<float>(R - H - zlo * sxj[j]);
            fhi[j] = static_cast<float>(H - 16 * zhi * sxj[j]);
          }
          const float vlo = fmaf(65536.f, flo[2], fmaf(256.f, flo[1], flo[0]));
          const float vhi = fmaf(65536.f, fhi[2], fmaf(256.f, fhi[1], fhi[0]));
          acc[w][m][0] = fmaf(vlo, sv[w][0] * pm, acc[w][m][0]);
          acc[w][m][1] = fmaf(vhi, sv[w][1] * (pm * 0.0625f), acc[w][m][1]);
        }
      }
      s += kI8Streams;
      if (s >= S) {
        s -= S;
        ph ^= 1;
      }
    }
  }

  // ---- reduction: the streams' partials in the drained ring, then per owner
  pdl_wait();   // y may still be read by the previous kernel
  cluster_wait_acquire();
  __syncthreads();
  float* red = reinterpret_cast<float*>(ring);  // [stream][token][256 columns]
  if (warp < kI8Consumers) {
    const int p = warp >> 1, tl = warp & 1;
    const int clo = (t >> 1) | ((t & 1) << 2);
#pragma unroll
    for (int m = 0; m < TOK; ++m)
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        float* rp = red + (p * TOK + m) * kI8Strip + 8 * (16 * tl + 2 * g + w) + clo;
        rp[0] = acc[w][m][0];
        rp[2] = acc[w][m][1];
      }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < kI8Strip; col += kI8Threads) {
    int r = C - 1;
    while (i8_col_lo(r, C) > col) --r;
    float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < TOK; ++m)
#pragma unroll
      for (int q = 0; q < kI8Streams; ++q) v4[m] += red[(q * TOK + m) * kI8Strip + col];
    const int li = col - i8_col_lo(r, C);
    st_async_v4(mapa_shared(smem_u32(recv + rank * cwmax + li), static_cast<uint32_t>(r)),
                make_float4(v4[0], v4[1], v4[2], v4[3]),
                mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r)));
  }
  const bool ok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
  if (ok) {
    for (int e = threadIdx.x; e < M * my_cols; e += kI8Threads) {
      const int m = e / my_cols, cl = e - m * my_cols;
      const int n = strip * kI8Strip + my_lo + cl;
      float v = 0.f;
      for (int q = 0; q < C; ++q) {
        const float4 r4 = recv[q * cwmax + cl];
        v += m == 0 ? r4.x : r4.y;
      }
      if (n < N) {
        if (bias != nullptr) v += Act<T>::to_float(bias[n]);
        y[static_cast<int64_t>(m) * N + n] = Act<T>::from_float(v);
      }
    }
  }
}

}  // namespace lmrs
