// decode_layer.cuh — one decoder layer of an FP8 (W8A8) decode step as ONE
// persistent kernel (lmrs_fp8_decode_layer).
//
// At decode batch sizes a tensor-parallel rank's layer is four weight streams
// (merged q/k/v, o, merged gate/up, down; ~107 MB of e4m3 at config 4, TP=8)
// and eight dependent small steps between them (norms, RoPE + KV write,
// attention, SiLU, the two all-reduces).  As separate kernels each dependent
// step costs a launch-to-launch latency of a few microseconds whatever its
// size, and every projection starts its weight stream cold.  Here one CTA per
// SM (a cooperative launch: all CTAs resident) runs the whole layer:
//   * warp 8 (one lane) streams this CTA's weight rows of all four projections,
//     in order, into a ring of shared-memory slots (16 rows x 2048 bytes of K:
//     ONE TMA box of a 3-D view [rows][K / 128][128] of the weight, L2
//     evict-first).  It never waits for activations, only for free slots, so
//     the next projection's weights flow in while the current phase's
//     dependencies resolve.  Measured on B200: one CTA's TMA boxes complete at
//     about one box per ~0.7 us, so the stream per SM grows with the box
//     (16 / 32 / 64 KB boxes: ~23 / ~26 / ~27 GB/s per SM at one CTA per SM,
//     against ~44 GB/s per SM for the whole HBM) and many small bulk copies
//     from one lane run slower still;
//   * warps 0-7 run the phases below, separated by grid-wide barriers (an
//     arrival counter that the last arriver resets and a generation word, in
//     the caller's workspace; every wait bounded);
//   * a projection's work is split into units of 16 weight rows x all of K
//     (one m16n8k32 e4m3 MMA tile of channels, the tokens as the MMA's 8
//     columns), assigned to CTAs on the host (lmrs_fp8_decode_layer_prepare)
//     so that every CTA's cumulative weight bytes stay balanced phase after
//     phase; within a slot warp w takes bytes [128 w, 128 w + 128) of K, and the
//     eight warps' partial sums meet in shared memory at the end of the unit.
// Phases (M tokens, H hidden, G = q heads per KV head):
//   R1  residual += the previous layer's down output (one rank: read; several:
//       the all-reduce packets the previous launch pushed, summed in rank order
//       and rounded as lmrs_allreduce_sum does), per-CTA column slices, partial
//       sums of squares                                                  | barrier
//   N1  RMSNorm(residual) * w_in rounded to bf16 into the row buffer, partial
//       absmax                                                           | barrier
//   Q   per-token e4m3 quantisation of the row (scale = absmax / 448, as
//       lmrs_fp8_quant_rows) into shared memory, the q/k/v units          | barrier
//   A   attention units (token, KV head, context chunk): RoPE of q and of the
//       new k (rope_pair), the new k / v written into the paged cache by the
//       unit that holds the position, scores, chunk softmax in the log2
//       domain, P V; (O, m, l) partials to the workspace                  | barrier
//   AM  merge of the chunks per (token, q head, 16 dims), bf16 output row,
//       partial absmax                                                   | barrier
//   O   quantised row, o units; one rank: bf16 output to the workspace
//       (barrier); several: each output pair pushed as an all-reduce packet
//       (data + flag in one 8-byte store) into every rank's receive buffer
//   R2  residual += the o output (local, or the packets: no barrier needed
//       before, the flags are the synchronisation)                        | barrier
//   N2  RMSNorm * w_post                                                 | barrier
//   GU  gate/up units                                                    | barrier
//   S   silu(gate) * up rounded to bf16 (as silu_mul_kernel), absmax       | barrier
//   D   down units: bf16 output (last layer / one rank) or all-reduce packets
//       for the next launch's R1.
// Arithmetic mirrors the separate kernels: the norm rounds once, the quantiser
// divides by the scale with IEEE division, projections accumulate in fp32 and
// apply s_x * s_w before one bf16 rounding, all-reduces sum in rank order.
// Summation orders inside the projections and the attention differ from the
// separate kernels, so results agree within fp32 accumulation noise, not bit
// for bit.
// The all-reduce packets use the lmrs_allreduce_sum buffers and epoch
// protocol (allreduce.cuh): with E the epoch at launch, R1 receives call E - 1,
// O pushes / R2 receives call E, D pushes call E + 1; the launch advances the
// epoch by 1 (+1 when D pushed), so the separate all-reduce kernels and this
// one can follow each other.
#pragma once
#include "allreduce.cuh"
#include "decode_ops.cuh"

namespace lmrs {

constexpr int kDlWarps = 8;                       // compute warps
constexpr int kDlThreads = 32 * (kDlWarps + 1);   // + the weight-stream warp
constexpr int kDlRows = 16;                       // weight rows per unit
#ifndef LMRS_DL_SEG
#define LMRS_DL_SEG 2048
#endif
constexpr int kDlSeg = LMRS_DL_SEG;               // K bytes per ring slot (one TMA box)
constexpr int kDlSlot = kDlRows * kDlSeg;         // [16 rows][kDlSeg / 128 K chunks][128 bytes]
constexpr int kDlMaxTok = 8;
constexpr int kDlMaxGroup = 8;                    // q heads per KV head
constexpr int kDlMaxChunk = 64;                   // context positions per attention unit
constexpr int kDlD = 128;                         // head size
constexpr int kDlMaxGrid = 256;
constexpr int kDlRedFloats = kDlWarps * kDlRows * kDlMaxTok;  // one unit's per-warp partials
constexpr int kDlMiscFloats = 768;
// attention scratch inside the shared "area": q [G][128] f32 | K, V tiles
// [64][128] bf16 | scores [G][64] f32
constexpr int kDlAttnQ = 0;
constexpr int kDlAttnK = kDlMaxGroup * kDlD * 4;
constexpr int kDlAttnV = kDlAttnK + kDlMaxChunk * kDlD * 2;
constexpr int kDlAttnS = kDlAttnV + kDlMaxChunk * kDlD * 2;
constexpr int kDlAttnBytes = kDlAttnS + kDlMaxGroup * kDlMaxChunk * 4;

enum { kDlQkv = 0, kDlO = 1, kDlGateUp = 2, kDlDown = 3 };

struct DlArgs {
  CUtensorMap tm[4];     // the weights as [N][K / 128][128] bytes, box [16][8][128]
  const uint8_t* w[4];   // e4m3 [N][K] row-major: qkv, o, gate_up, down
  const float* sw[4];    // fp32 [N] per-channel scales
  int N[4], K[4];
  const __nv_bfloat16* in_norm;
  const __nv_bfloat16* post_norm;
  __nv_bfloat16* kc;     // [blocks][hkv][block_size][128]
  __nv_bfloat16* vc;
  const int32_t* tables; // [M][max_blocks]
  const int32_t* ctx_lens;
  const __nv_bfloat16* cosv;  // [64]
  const __nv_bfloat16* sinv;
  __nv_bfloat16* resid;        // [M][H], in place
  const __nv_bfloat16* delta_in;
  __nv_bfloat16* delta_out;
  int M, H, hq, hkv, inter, block_size, max_blocks, chunk, nchunk, ring, area;
  float eps, scale_log2;
  int rank, world, recv_delta, push_delta, cap;
  ArPeers peers;
  // workspace
  unsigned long long* bar;  // grid-barrier arrival counter (only grows)
  float* st_ss;          // [grid][8] per-CTA sums of squares of the residual slices
  float* st_max;         // [grid][8] per-CTA absmax of the next projection's input slices
  const int* sched;      // [4][grid + 1] offsets, then the unit list
  __nv_bfloat16* xrow;   // [M][K of the next projection]
  __nv_bfloat16* qkv;    // [M][N qkv]
  __nv_bfloat16* gu;     // [M][2 inter]
  __nv_bfloat16* obuf;   // [M][H]
  float* att_o;          // [M][hkv][nchunk][G][128]
  float* att_ml;         // [M][hkv][nchunk][G][2]
  unsigned long long* trace;  // optional [grid][32] phase timestamps (ns), or null
};

constexpr int kDlTraceSlots = 32;

// Phase trace: thread 0 of each CTA stores the global timer into its next slot.
__device__ __forceinline__ void dl_mark(const DlArgs& a, int& mk) {
  if (a.trace != nullptr && threadIdx.x == 0 && mk < kDlTraceSlots) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.trace[blockIdx.x * kDlTraceSlots + mk] = t;
  }
  ++mk;
}

__host__ __device__ constexpr int dl_smem_bytes(int ring, int area) {
  return 1024 + ring * kDlSlot + area + 2 * kDlRedFloats * 4 + kDlMiscFloats * 4 + 2 * ring * 8;
}

__device__ __forceinline__ void dl_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ unsigned long long dl_ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void dl_red_release(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Ring-slot wait for a CTA that is alone on its SM: spin on test_wait (a
// suspended waiter's wake-up is not hidden by other CTAs here); bounded.
__device__ __forceinline__ bool dl_mbar_spin(uint64_t* bar, uint32_t parity, uint32_t site) {
  auto test = [&]() {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
  };
  if (test()) return true;
  const long long t0 = clock64();
  long long limit = -1;
  while (!test()) {
    if (wait_expired(t0, limit)) {
      atomicOr(&g_device_error, site);
      return false;
    }
  }
  return true;
}

// 3-D tiled TMA load (no multicast), completion counted on `bar`.
__device__ __forceinline__ void dl_tma_load_3d(const CUtensorMap* m, uint64_t* bar, void* dst,
                                               int32_t c0, int32_t c1, int32_t c2,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint4 dl_ldcg4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// Grid-wide barrier of the compute warps of every CTA, on a 64-bit arrival
// counter that only grows: every barrier adds `grid` to it, so barrier k of a
// launch completes when it reaches base + (k + 1) x grid, base = its value at
// launch rounded down to a multiple of the grid (only arrivals at the first
// barrier can precede that read).  An arrival is one fire-and-forget
// red.release; no reset round trip.  Thread 0 of each CTA holds `target`.
__device__ __forceinline__ void dl_grid_sync(unsigned long long* ctr, unsigned long long& target,
                                             bool& ok) {
  dl_bar_sync();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    dl_red_release(ctr, 1ull);
    if (ok && dl_ld_acquire(ctr) < target) {
      const long long t0 = clock64();
      long long limit = -1;
      while (dl_ld_acquire(ctr) < target) {
        if (wait_expired(t0, limit)) {
          atomicOr(&g_device_error, kErrWaitGrid);
          ok = false;
          break;
        }
      }
    }
  }
  dl_bar_sync();
}

// Per-token reduction over the 256 compute threads: v[m] for m < M ->
// out[m] (shared).  Fixed order: the same in every CTA.
template <bool MAX>
__device__ __forceinline__ void dl_reduce8(float (&v)[kDlMaxTok], int M, float* wred,
                                           float* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 0; m < kDlMaxTok; ++m) {
    if (m >= M) break;
    float x = v[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, x, o);
      x = MAX ? fmaxf(x, y) : x + y;
    }
    if (lane == 0) wred[warp * kDlMaxTok + m] = x;
  }
  dl_bar_sync();
  if (threadIdx.x < M) {
    float r = wred[threadIdx.x];
    for (int w = 1; w < kDlWarps; ++w) {
      const float y = wred[w * kDlMaxTok + threadIdx.x];
      r = MAX ? fmaxf(r, y) : r + y;
    }
    out[threadIdx.x] = r;
  }
  dl_bar_sync();
}

// out[m] = sum (or max) over the grid's CTAs of parts[cta][m], in CTA order.
template <bool MAX>
__device__ __forceinline__ void dl_grid_stat(const float* parts, int M, float* wred, float* out) {
  float v[kDlMaxTok];
#pragma unroll
  for (int m = 0; m < kDlMaxTok; ++m)
    v[m] = (threadIdx.x < gridDim.x && m < M) ? __ldcg(parts + threadIdx.x * kDlMaxTok + m) : 0.f;
  dl_reduce8<MAX>(v, M, wred, out);
}

// This CTA's slice [lo, hi) of n 8-element vectors.
__device__ __forceinline__ void dl_slice(int n, int& lo, int& hi) {
  lo = static_cast<int>((static_cast<long long>(blockIdx.x) * n) / gridDim.x);
  hi = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * n) / gridDim.x);
}

// Sum over the ranks, in rank order, of the packets holding elements
// [2 i2, 2 i2 + 8) of one all-reduce call; rounded to bf16 as the all-reduce
// kernels do.  A source whose packets never arrive gives NaN.
__device__ __forceinline__ uint4 dl_packets8(const DlArgs& a, int64_t i2, uint32_t flagv,
                                             int phase, bool& ok) {
  const uint64_t flag = static_cast<uint64_t>(flagv) << 32;
  const uint64_t* own = a.peers.buf[a.rank] + static_cast<int64_t>(phase) * a.world * a.cap + i2;
  uint64_t pk[kArMaxRanks][4];
#pragma unroll
  for (int s = 0; s < kArMaxRanks; ++s)
    if (s < a.world)
#pragma unroll
      for (int j = 0; j < 4; ++j) pk[s][j] = ld_sys_b64_once(own + static_cast<int64_t>(s) * a.cap + j);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < kArMaxRanks; ++s) {
    if (s >= a.world) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint64_t p = pk[s][j];
      if ((p & 0xFFFFFFFF00000000ull) != flag) {
        const uint64_t* src = own + static_cast<int64_t>(s) * a.cap + j;
        const long long t0 = clock64();
        long long limit = -1;
        while (ok && ((p = ld_sys_b64(src)) & 0xFFFFFFFF00000000ull) != flag) {
          if (wait_expired(t0, limit)) {
            atomicOr(&g_device_error, kErrWaitPeer);
            ok = false;
          }
        }
      }
      if ((p & 0xFFFFFFFF00000000ull) != flag) {
        acc[2 * j] = acc[2 * j + 1] = __int_as_float(0x7fc00000);
      } else {
        const float2 f = Act<__nv_bfloat16>::unpack2(static_cast<uint32_t>(p));
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
  }
  return make_uint4(Act<__nv_bfloat16>::pack2(acc[0], acc[1]), Act<__nv_bfloat16>::pack2(acc[2], acc[3]),
                    Act<__nv_bfloat16>::pack2(acc[4], acc[5]), Act<__nv_bfloat16>::pack2(acc[6], acc[7]));
}

// Eight bf16 values: x + d rounded (the residual add of rmsnorm_kernel), sum
// of squares, absmax, and RMSNorm x * rstd * w rounded once.
__device__ __forceinline__ uint4 dl_add8(const uint4& x, const uint4& d) {
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x);
  const uint32_t* dw = reinterpret_cast<const uint32_t*>(&d);
  uint4 r;
  uint32_t* rw = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = Act<__nv_bfloat16>::unpack2(xw[i]), q = Act<__nv_bfloat16>::unpack2(dw[i]);
    rw[i] = Act<__nv_bfloat16>::pack2(p.x + q.x, p.y + q.y);
  }
  return r;
}
__device__ __forceinline__ float dl_ss8(const uint4& x) {
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = Act<__nv_bfloat16>::unpack2(xw[i]);
    s += p.x * p.x;
    s += p.y * p.y;
  }
  return s;
}
__device__ __forceinline__ float dl_amax8(const uint4& x) {
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = Act<__nv_bfloat16>::unpack2(xw[i]);
    s = fmaxf(s, fmaxf(fabsf(p.x), fabsf(p.y)));
  }
  return s;
}
__device__ __forceinline__ uint4 dl_norm8(const uint4& x, const uint4& w, float inv) {
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x);
  const uint32_t* ww = reinterpret_cast<const uint32_t*>(&w);
  uint4 r;
  uint32_t* rw = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = Act<__nv_bfloat16>::unpack2(xw[i]), g = Act<__nv_bfloat16>::unpack2(ww[i]);
    rw[i] = Act<__nv_bfloat16>::pack2(p.x * inv * g.x, p.y * inv * g.y);
  }
  return r;
}

// R: residual += delta over this CTA's column slice (src 0: none, 1: a bf16
// array, 2: the all-reduce packets of call (flagv, phase)), then the slice's
// sums of squares per token.
__device__ void dl_residual(const DlArgs& a, int src, const __nv_bfloat16* dloc, uint32_t flagv,
                            int phase, float* wred, float* scratch, bool& ok) {
  int lo, hi;
  dl_slice(a.H / 8, lo, hi);
  float ss[kDlMaxTok];
#pragma unroll
  for (int m = 0; m < kDlMaxTok; ++m) ss[m] = 0.f;
  for (int v = lo + static_cast<int>(threadIdx.x); v < hi; v += 256) {
    uint4 hv[kDlMaxTok], dv[kDlMaxTok];
#pragma unroll
    for (int m = 0; m < kDlMaxTok; ++m)  // every token's loads in flight together
      if (m < a.M) {
        const int64_t off = static_cast<int64_t>(m) * a.H + v * 8;
        hv[m] = dl_ldcg4(a.resid + off);
        if (src == 1) dv[m] = dl_ldcg4(dloc + off);
      }
#pragma unroll
    for (int m = 0; m < kDlMaxTok; ++m) {
      if (m >= a.M) break;
      const int64_t off = static_cast<int64_t>(m) * a.H + v * 8;
      if (src != 0) {
        if (src == 2) dv[m] = dl_packets8(a, off / 2, flagv, phase, ok);
        hv[m] = dl_add8(hv[m], dv[m]);
        *reinterpret_cast<uint4*>(a.resid + off) = hv[m];
      }
      ss[m] += dl_ss8(hv[m]);
    }
  }
  dl_reduce8<false>(ss, a.M, wred, scratch);
  if (threadIdx.x < a.M) a.st_ss[blockIdx.x * kDlMaxTok + threadIdx.x] = scratch[threadIdx.x];
}

// N: row buffer = RMSNorm(residual) * w (rounded once) over this CTA's slice,
// with the rstd from every CTA's sums of squares; the slice's absmax.
__device__ void dl_norm(const DlArgs& a, const __nv_bfloat16* w, float* wred, float* scratch) {
  dl_grid_stat<false>(a.st_ss, a.M, wred, scratch);
  float inv[kDlMaxTok];
#pragma unroll
  for (int m = 0; m < kDlMaxTok; ++m) inv[m] = m < a.M ? rsqrtf(scratch[m] / a.H + a.eps) : 0.f;
  int lo, hi;
  dl_slice(a.H / 8, lo, hi);
  float amax[kDlMaxTok];
#pragma unroll
  for (int m = 0; m < kDlMaxTok; ++m) amax[m] = 0.f;
  for (int v = lo + static_cast<int>(threadIdx.x); v < hi; v += 256) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + v * 8));
    uint4 hvs[kDlMaxTok];
#pragma unroll
    for (int m = 0; m < kDlMaxTok; ++m)
      if (m < a.M) hvs[m] = dl_ldcg4(a.resid + static_cast<int64_t>(m) * a.H + v * 8);
#pragma unroll
    for (int m = 0; m < kDlMaxTok; ++m) {
      if (m >= a.M) break;
      const uint4 y = dl_norm8(hvs[m], wv, inv[m]);
      amax[m] = fmaxf(amax[m], dl_amax8(y));
      *reinterpret_cast<uint4*>(a.xrow + static_cast<int64_t>(m) * a.H + v * 8) = y;
    }
  }
  dl_reduce8<true>(amax, a.M, wred, scratch);
  if (threadIdx.x < a.M) a.st_max[blockIdx.x * kDlMaxTok + threadIdx.x] = scratch[threadIdx.x];
}

// S: row buffer = silu(gate) * up rounded as silu_mul_kernel, slice absmax.
__device__ void dl_silu(const DlArgs& a, float* wred, float* scratch) {
  int lo, hi;
  dl_slice(a.inter / 8, lo, hi);
  float amax[kDlMaxTok];
#pragma unroll
  for (int m = 0; m < kDlMaxTok; ++m) amax[m] = 0.f;
  for (int v = lo + static_cast<int>(threadIdx.x); v < hi; v += 256) {
    uint4 gv[kDlMaxTok], uv[kDlMaxTok];
#pragma unroll
    for (int m = 0; m < kDlMaxTok; ++m)
      if (m < a.M) {
        const __nv_bfloat16* gr = a.gu + static_cast<int64_t>(m) * 2 * a.inter + v * 8;
        gv[m] = dl_ldcg4(gr);
        uv[m] = dl_ldcg4(gr + a.inter);
      }
#pragma unroll
    for (int m = 0; m < kDlMaxTok; ++m) {
      if (m >= a.M) break;
      float g[8], u[8];
      unpack8<__nv_bfloat16>(gv[m], g);
      unpack8<__nv_bfloat16>(uv[m], u);
      uint4 ov;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
      for (int i = 0; i < 8; ++i) oe[i] = __float2bfloat16_rn((g[i] / (1.0f + expf(-g[i]))) * u[i]);
      amax[m] = fmaxf(amax[m], dl_amax8(ov));
      *reinterpret_cast<uint4*>(a.xrow + static_cast<int64_t>(m) * a.inter + v * 8) = ov;
    }
  }
  dl_reduce8<true>(amax, a.M, wred, scratch);
  if (threadIdx.x < a.M) a.st_max[blockIdx.x * kDlMaxTok + threadIdx.x] = scratch[threadIdx.x];
}

// One projection phase of the compute warps: quantise the row buffer (this
// phase's input, [M][K]) into shared memory, then this CTA's units.  Output
// pairs go to `out` ([M][N] bf16) and/or, as all-reduce packets of call
// (flagv, phase), to every rank.
__device__ void dl_gemv(const DlArgs& a, int p, uint8_t* ring, uint8_t* xq, float* red,
                        float* wred, float* sx, uint64_t* full, uint64_t* empty, uint32_t& it,
                        uint32_t& ucount, __nv_bfloat16* out, bool push, uint32_t flagv,
                        int phase, bool& ok, int& mk) {
  const int G = static_cast<int>(gridDim.x);
  const int beg = a.sched[p * (G + 1) + blockIdx.x], end = a.sched[p * (G + 1) + blockIdx.x + 1];
  if (beg >= end) {
    dl_mark(a, mk);
    return;
  }
  const int* units = a.sched + 4 * (G + 1);
  const int K = a.K[p], N = a.N[p], XP = K + 16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;

  dl_grid_stat<true>(a.st_max, a.M, wred, sx);
  if (tid < a.M) sx[tid] = __fdiv_rn(sx[tid], 448.0f);
  dl_bar_sync();
  {  // the row buffer is [M][K] contiguous: vector e = (m, k8) sits at 8 e
    const int nv = K / 8, tot = a.M * nv;
    for (int e0 = tid; e0 < tot; e0 += 256 * 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (e0 + j * 256 < tot) v[j] = dl_ldcg4(a.xrow + static_cast<int64_t>(e0 + j * 256) * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = e0 + j * 256;
        if (e < tot) {
          const int m = e / nv, k8 = e - m * nv;
          float f[8];
          unpack8<__nv_bfloat16>(v[j], f);
          *reinterpret_cast<uint2*>(xq + m * XP + k8 * 8) = e4m3x8(f, sx[m]);
        }
      }
    }
  }
  dl_bar_sync();
  dl_mark(a, mk);  // input row quantised

  const uint64_t flag = static_cast<uint64_t>(flagv) << 32;
  for (int ui = beg; ui < end; ++ui) {
    const int row0 = units[ui] * kDlRows;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // the epilogue threads' channel scales, loaded before the unit's MMAs
    float2 swp = make_float2(0.f, 0.f);
    if (tid < 64) swp = __ldg(reinterpret_cast<const float2*>(a.sw[p] + row0 + 2 * (tid >> 3)));
    for (int k0 = 0; k0 < K; k0 += kDlSeg) {
      const int slot = static_cast<int>(it % static_cast<uint32_t>(a.ring));
      const uint32_t par = (it / static_cast<uint32_t>(a.ring)) & 1u;
      if (!dl_mbar_spin(&full[slot], par, kErrWaitFull)) ok = false;
      const int len = K - k0 < kDlSeg ? K - k0 : kDlSeg;
#pragma unroll
      for (int j = warp; j < kDlSeg / 128; j += kDlWarps) {  // this warp's 128-byte K chunks
        if (j * 128 >= len) break;
        const uint8_t* sb = ring + slot * kDlSlot + j * 128;  // row r at r * kDlSeg
        const uint4 ga = *reinterpret_cast<const uint4*>(sb + g * kDlSeg + 16 * t);
        const uint4 gc = *reinterpret_cast<const uint4*>(sb + g * kDlSeg + 64 + 16 * t);
        const uint4 ha = *reinterpret_cast<const uint4*>(sb + (g + 8) * kDlSeg + 16 * t);
        const uint4 hc = *reinterpret_cast<const uint4*>(sb + (g + 8) * kDlSeg + 64 + 16 * t);
        uint4 xa = make_uint4(0u, 0u, 0u, 0u), xc = xa;
        if (g < a.M) {
          const uint8_t* xr = xq + g * XP + k0 + j * 128;
          xa = *reinterpret_cast<const uint4*>(xr + 16 * t);
          xc = *reinterpret_cast<const uint4*>(xr + 64 + 16 * t);
        }
        mma_e4m3_16832(acc, ga.x, ha.x, ga.y, ha.y, xa.x, xa.y);
        mma_e4m3_16832(acc, ga.z, ha.z, ga.w, ha.w, xa.z, xa.w);
        mma_e4m3_16832(acc, gc.x, hc.x, gc.y, hc.y, xc.x, xc.y);
        mma_e4m3_16832(acc, gc.z, hc.z, gc.w, hc.w, xc.z, xc.w);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      ++it;
    }
    float* r = red + (ucount & 1u) * kDlRedFloats;  // [warp][row][token]
    r[(warp * kDlRows + g) * kDlMaxTok + 2 * t] = acc[0];
    r[(warp * kDlRows + g) * kDlMaxTok + 2 * t + 1] = acc[1];
    r[(warp * kDlRows + g + 8) * kDlMaxTok + 2 * t] = acc[2];
    r[(warp * kDlRows + g + 8) * kDlMaxTok + 2 * t + 1] = acc[3];
    dl_bar_sync();
    if (tid < 64) {
      const int rp = tid >> 3, m = tid & 7;
      if (m < a.M) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int w = 0; w < kDlWarps; ++w) {
          s0 += r[(w * kDlRows + 2 * rp) * kDlMaxTok + m];
          s1 += r[(w * kDlRows + 2 * rp + 1) * kDlMaxTok + m];
        }
        const int n = row0 + 2 * rp;
        const float v0 = __fmul_rn(__fmul_rn(s0, sx[m]), swp.x);
        const float v1 = __fmul_rn(__fmul_rn(s1, sx[m]), swp.y);
        const uint32_t pair = Act<__nv_bfloat16>::pack2(v0, v1);
        const int64_t idx = static_cast<int64_t>(m) * N + n;
        if (out != nullptr) *reinterpret_cast<uint32_t*>(out + idx) = pair;
        if (push) {
          const uint64_t pkt = flag | pair;
          for (int q = 0; q < a.world; ++q)
            st_sys_b64(a.peers.buf[q] + (static_cast<int64_t>(phase) * a.world + a.rank) * a.cap + idx / 2,
                       pkt);
        }
      }
    }
    ++ucount;
  }
}

// A: attention units (token, KV head, chunk of the context).  Two passes of
// global loads per unit: (1) the raw q rows, cos / sin, the new k and v (the
// unit holding the new position) and the chunk's block ids; (2) the chunk's K
// and V rows into registers, issued before the RoPE of q and k so that the
// rotation hides their latency.  The new token's row of the tile comes from
// the rotated k / raw v in shared memory, and that unit writes them into the
// cache (so no unit reads back a cache write of this launch).
__device__ void dl_attention(const DlArgs& a, uint8_t* area, float* misc, int& mk) {
  const int G = a.hq / a.hkv, L = a.chunk, nch = a.nchunk, Nq = a.N[kDlQkv];
  const int bs = a.block_size;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* sq = reinterpret_cast<float*>(area + kDlAttnQ);
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(area + kDlAttnK);
  __nv_bfloat16* sv = reinterpret_cast<__nv_bfloat16*>(area + kDlAttnV);
  float* sc = reinterpret_cast<float*>(area + kDlAttnS);
  __nv_bfloat16* qraw = reinterpret_cast<__nv_bfloat16*>(sc);  // until the scores overwrite it
  __nv_bfloat16* kn = reinterpret_cast<__nv_bfloat16*>(misc + 384);
  __nv_bfloat16* vn = reinterpret_cast<__nv_bfloat16*>(misc + 448);
  __nv_bfloat16* cs = reinterpret_cast<__nv_bfloat16*>(misc + 512);  // cos [64] | sin [64]
  int* sblk = reinterpret_cast<int*>(misc + 576);                     // <= 64 / bs + 2 ids
  const int units = a.M * a.hkv * nch;
  const int cap_ctx = a.max_blocks * bs;
  if (static_cast<int>(blockIdx.x) >= units) mk += 2;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int m = u / (a.hkv * nch), kvh = (u / nch) % a.hkv, c = u % nch;
    int ctx = a.ctx_lens[m];
    ctx = ctx < 0 ? 0 : (ctx > cap_ctx ? cap_ctx : ctx);
    const int p0 = c * L;
    const int p1 = p0 + L < ctx ? p0 + L : ctx;
    const int np = p1 > p0 ? p1 - p0 : 0;
    const int pos = ctx - 1;
    const bool owner = pos >= p0 && pos < p1;
    const int b0 = p0 / bs;
    const int nb = np > 0 ? (p1 - 1) / bs - b0 + 1 : 0;
    const __nv_bfloat16* row = a.qkv + static_cast<int64_t>(m) * Nq;
    // load pass 1
    const int nq = G * 16, nown = owner ? 32 : 0, n1 = nq + 16 + nown + nb;
    for (int i = tid; i < n1; i += 256) {
      if (i < nq) {
        const int g = i >> 4, ch = i & 15;
        *reinterpret_cast<uint4*>(qraw + g * kDlD + ch * 8) = dl_ldcg4(row + (kvh * G + g) * kDlD + ch * 8);
      } else if (i < nq + 16) {
        const int j = i - nq;
        *reinterpret_cast<uint4*>(cs + j * 8) =
            __ldg(reinterpret_cast<const uint4*>(j < 8 ? a.cosv + j * 8 : a.sinv + (j - 8) * 8));
      } else if (i < nq + 16 + nown) {
        const int j = i - nq - 16;
        if (j < 16)
          *reinterpret_cast<uint4*>(kn + j * 8) = dl_ldcg4(row + (a.hq + kvh) * kDlD + j * 8);
        else
          *reinterpret_cast<uint4*>(vn + (j - 16) * 8) =
              dl_ldcg4(row + (a.hq + a.hkv + kvh) * kDlD + (j - 16) * 8);
      } else {
        const int j = i - nq - 16 - nown;
        sblk[j] = __ldg(a.tables + static_cast<int64_t>(m) * a.max_blocks + b0 + j);
      }
    }
    dl_bar_sync();
    if (u == static_cast<int>(blockIdx.x)) dl_mark(a, mk);  // first unit: load pass 1 in
    // load pass 2: K / V rows into registers (np * 16 <= 1024 vectors: 4 per thread)
    uint4 kr[4], vr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = tid + j * 256;
      kr[j] = vr[j] = make_uint4(0u, 0u, 0u, 0u);
      if (e < np * 16) {
        const int p = p0 + (e >> 4), ch = e & 15;
        if (p != pos) {
          const int64_t off =
              ((static_cast<int64_t>(sblk[p / bs - b0]) * a.hkv + kvh) * bs + p % bs) * kDlD + ch * 8;
          kr[j] = dl_ldcg4(a.kc + off);
          vr[j] = dl_ldcg4(a.vc + off);
        }
      }
    }
    // RoPE of q (fp32 of the bf16-rounded rotation, as the attention kernels feed
    // it to their MMAs) and of the new k (in place)
    for (int idx = tid; idx < G * 64; idx += 256) {
      const int g = idx >> 6, i = idx & 63;
      const float2 r = rope_pair(__bfloat162float(qraw[g * kDlD + i]), __bfloat162float(qraw[g * kDlD + i + 64]),
                                 __bfloat162float(cs[i]), __bfloat162float(cs[64 + i]));
      sq[g * kDlD + i] = __bfloat162float(__float2bfloat16_rn(r.x));
      sq[g * kDlD + i + 64] = __bfloat162float(__float2bfloat16_rn(r.y));
    }
    if (owner && tid < 64) {
      const float2 r = rope_pair(__bfloat162float(kn[tid]), __bfloat162float(kn[tid + 64]),
                                 __bfloat162float(cs[tid]), __bfloat162float(cs[64 + tid]));
      kn[tid] = __float2bfloat16_rn(r.x);
      kn[tid + 64] = __float2bfloat16_rn(r.y);
    }
    dl_bar_sync();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = tid + j * 256;
      if (e < np * 16) {
        const int p = p0 + (e >> 4), ch = e & 15;
        const bool own = p == pos;
        *reinterpret_cast<uint4*>(sk + (p - p0) * kDlD + ch * 8) =
            own ? *reinterpret_cast<const uint4*>(kn + ch * 8) : kr[j];
        *reinterpret_cast<uint4*>(sv + (p - p0) * kDlD + ch * 8) =
            own ? *reinterpret_cast<const uint4*>(vn + ch * 8) : vr[j];
      }
    }
    if (owner && tid < 32) {
      const int64_t off =
          ((static_cast<int64_t>(sblk[pos / bs - b0]) * a.hkv + kvh) * bs + pos % bs) * kDlD;
      if (tid < 16)
        *reinterpret_cast<uint4*>(a.kc + off + tid * 8) = *reinterpret_cast<const uint4*>(kn + tid * 8);
      else
        *reinterpret_cast<uint4*>(a.vc + off + (tid - 16) * 8) =
            *reinterpret_cast<const uint4*>(vn + (tid - 16) * 8);
    }
    dl_bar_sync();
    if (u == static_cast<int>(blockIdx.x)) dl_mark(a, mk);  // first unit: tile in shared memory
    // scores: 8 lanes per position (16 dims each), 4 positions per warp and step,
    // 3-step shuffle sums within the 8 lanes; the heads' sums are independent
    for (int pw = warp * 4; pw < np; pw += kDlWarps * 4) {
      const int p = pw + (lane >> 3), db = lane & 7;
      float kf[16];
      if (p < np) {
        const uint4 k0 = *reinterpret_cast<const uint4*>(sk + p * kDlD + 16 * db);
        const uint4 k1 = *reinterpret_cast<const uint4*>(sk + p * kDlD + 16 * db + 8);
        unpack8<__nv_bfloat16>(k0, *reinterpret_cast<float(*)[8]>(&kf[0]));
        unpack8<__nv_bfloat16>(k1, *reinterpret_cast<float(*)[8]>(&kf[8]));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) kf[i] = 0.f;
      }
#pragma unroll
      for (int gq = 0; gq < kDlMaxGroup; ++gq) {
        if (gq >= G) break;
        const float4* qv = reinterpret_cast<const float4*>(sq + gq * kDlD + 16 * db);
        float sdot = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 q = qv[i];
          sdot += q.x * kf[4 * i] + q.y * kf[4 * i + 1] + q.z * kf[4 * i + 2] + q.w * kf[4 * i + 3];
        }
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 4);
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
        if (p < np && db == 0) sc[gq * kDlMaxChunk + p] = sdot * a.scale_log2;
      }
    }
    dl_bar_sync();
    if (warp < G) {
      float* srow = sc + warp * kDlMaxChunk;
      float mx = -INFINITY;
      for (int p = lane; p < np; p += 32) mx = fmaxf(mx, srow[p]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float l = 0.f;
      for (int p = lane; p < np; p += 32) {
        const float e = exp2f(srow[p] - mx);
        srow[p] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      __syncwarp();
      float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < np; ++p) {
        const float pe = srow[p];
        const uint2 vr2 = *reinterpret_cast<const uint2*>(sv + p * kDlD + 4 * lane);
        const float2 v01 = Act<__nv_bfloat16>::unpack2(vr2.x), v23 = Act<__nv_bfloat16>::unpack2(vr2.y);
        o4.x += pe * v01.x;
        o4.y += pe * v01.y;
        o4.z += pe * v23.x;
        o4.w += pe * v23.y;
      }
      const int64_t pi = static_cast<int64_t>(u) * G + warp;
      *reinterpret_cast<float4*>(a.att_o + pi * kDlD + 4 * lane) = o4;
      if (lane == 0) {
        a.att_ml[pi * 2] = mx;
        a.att_ml[pi * 2 + 1] = l;
      }
    }
    dl_bar_sync();
  }
}

// AM: merge the chunks of each (token, q head) for 16 dims per unit: 16
// chunk groups x 16 dims over the CTA, each thread one pass over its chunks
// (eight chunks' (m, l, o) loads in flight, running maximum with rescaling),
// then the 16 groups combined in order; bf16 attention row into the row
// buffer, this CTA's absmax.
__device__ void dl_attn_merge(const DlArgs& a, float* misc) {
  const int G = a.hq / a.hkv, nch = a.nchunk;
  const int tid = threadIdx.x;
  const int cg = tid >> 4, dl = tid & 15;
  float* sO = misc;                  // [16 groups][16 dims]
  float* sl = misc + 256;            // [16]
  float* smx = misc + 272;           // [16]
  float* amx = misc + 368;           // [8] this CTA's absmax per token
  if (tid < kDlMaxTok) amx[tid] = 0.f;
  const int units = a.M * a.hq * 8;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int m = u / (a.hq * 8), h = (u >> 3) % a.hq, slc = u & 7;
    const int kvh = h / G, gq = h % G;
    const int d = slc * 16 + dl;
    const int64_t base = static_cast<int64_t>(m * a.hkv + kvh) * nch;
    float mx = -INFINITY, o = 0.f, l = 0.f;
    for (int c0 = cg; c0 < nch; c0 += 16 * 8) {
      float mv[8], lv[8], ov[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + 16 * j;
        const int64_t pi = (base + (c < nch ? c : 0)) * G + gq;
        mv[j] = c < nch ? __ldcg(a.att_ml + pi * 2) : -INFINITY;
        lv[j] = __ldcg(a.att_ml + pi * 2 + 1);
        ov[j] = __ldcg(a.att_o + pi * kDlD + d);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (mv[j] == -INFINITY) continue;  // an empty chunk (or none)
        if (mv[j] > mx) {
          const float r = exp2f(mx - mv[j]);
          o *= r;
          l *= r;
          mx = mv[j];
        }
        const float w = exp2f(mv[j] - mx);
        o += w * ov[j];
        l += w * lv[j];
      }
    }
    sO[cg * 16 + dl] = o;
    if (dl == 0) {
      sl[cg] = l;
      smx[cg] = mx;
    }
    dl_bar_sync();
    if (tid < 16) {
      float Mx = -INFINITY;
      for (int q = 0; q < 16; ++q) Mx = fmaxf(Mx, smx[q]);
      float O = 0.f, Lt = 0.f;
      if (Mx != -INFINITY)
        for (int q = 0; q < 16; ++q) {
          if (smx[q] == -INFINITY) continue;
          const float w = exp2f(smx[q] - Mx);
          O += w * sO[q * 16 + tid];
          Lt += w * sl[q];
        }
      const __nv_bfloat16 b = __float2bfloat16_rn(Lt > 0.f ? O / Lt : 0.f);
      a.xrow[static_cast<int64_t>(m) * a.hq * kDlD + h * kDlD + slc * 16 + tid] = b;
      float am = fabsf(__bfloat162float(b));
#pragma unroll
      for (int q = 8; q > 0; q >>= 1) am = fmaxf(am, __shfl_xor_sync(0x0000ffffu, am, q));
      if (tid == 0) amx[m] = fmaxf(amx[m], am);
    }
    dl_bar_sync();
  }
  if (tid < a.M) a.st_max[blockIdx.x * kDlMaxTok + tid] = amx[tid];
}

__global__ void __launch_bounds__(kDlThreads, 1) fp8_decode_layer_kernel(const __grid_constant__ DlArgs a) {
  extern __shared__ uint8_t dl_smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dl_smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* area = ring + a.ring * kDlSlot;
  float* red = reinterpret_cast<float*>(area + a.area);
  float* misc = red + 2 * kDlRedFloats;
  uint64_t* full = reinterpret_cast<uint64_t*>(misc + kDlMiscFloats);
  uint64_t* empty = full + a.ring;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = static_cast<int>(gridDim.x);

  if (tid == 0) {
    for (int s = 0; s < a.ring; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDlWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kDlWarps) {  // ---- weight stream
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int p = 0; p < 4; ++p) tma_prefetch_desc(&a.tm[p]);
      const int* units = a.sched + 4 * (G + 1);
      uint32_t it = 0;
      bool live = true;
      for (int p = 0; p < 4 && live; ++p) {
        const int beg = a.sched[p * (G + 1) + blockIdx.x], end = a.sched[p * (G + 1) + blockIdx.x + 1];
        const int K = a.K[p];
        for (int ui = beg; ui < end && live; ++ui) {
          const int row0 = units[ui] * kDlRows;
          for (int k0 = 0; k0 < K; k0 += kDlSeg) {
            const int slot = static_cast<int>(it % static_cast<uint32_t>(a.ring));
            if (it >= static_cast<uint32_t>(a.ring) &&
                !dl_mbar_spin(&empty[slot], ((it / static_cast<uint32_t>(a.ring)) - 1u) & 1u,
                              kErrWaitEmpty)) {
              live = false;
              break;
            }
            // a box past K is zero-filled and still counts its full bytes
            mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(kDlSlot));
            dl_tma_load_3d(&a.tm[p], &full[slot], ring + slot * kDlSlot, 0, k0 / 128, row0, pol);
            ++it;
          }
        }
      }
    }
    return;
  }

  // ---- compute warps
  // phase trace (lmrs_set_tuning "decode_layer_trace"): global timer at the
  // start, and before and after every grid barrier, one row of slots per CTA
  int mk = 0;
  auto mark = [&]() { dl_mark(a, mk); };
  mark();
  // misc: [0, 288) merge scratch | wred [8 warps][8 tokens] | scratch [8] | sx [8] |
  // merge absmax [8] | kn, vn (bf16 [128] each) | cos | sin | block ids
  float* wred = misc + 288;
  float* scratch = misc + 352;
  float* sx = misc + 360;
  bool ok = true;
  uint32_t it = 0, ucount = 0;
  unsigned long long target = 0;
  if (tid == 0) {
    const unsigned long long v = dl_ld_acquire(a.bar);
    target = v - v % static_cast<unsigned long long>(G);
  }
  const bool tp = a.world > 1;
  uint32_t* ctrl = tp ? reinterpret_cast<uint32_t*>(a.peers.buf[a.rank]) - 16 : nullptr;
  const uint32_t E = tp ? *reinterpret_cast<volatile uint32_t*>(ctrl) : 0u;

  const int src1 = tp ? (a.recv_delta ? 2 : 0) : (a.delta_in != nullptr ? 1 : 0);
  dl_residual(a, src1, a.delta_in, E, static_cast<int>((E - 1u) & 1u), wred, scratch, ok);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_norm(a, a.in_norm, wred, scratch);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_gemv(a, kDlQkv, ring, area, red, wred, sx, full, empty, it, ucount, a.qkv, false, 0u, 0, ok, mk);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_attention(a, area, misc, mk);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_attn_merge(a, misc);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_gemv(a, kDlO, ring, area, red, wred, sx, full, empty, it, ucount, tp ? nullptr : a.obuf, tp,
          E + 1u, static_cast<int>(E & 1u), ok, mk);
  mark();
  if (!tp) dl_grid_sync(a.bar, target, ok);  // several ranks: the packet flags order R2
  mark();
  dl_residual(a, tp ? 2 : 1, a.obuf, E + 1u, static_cast<int>(E & 1u), wred, scratch, ok);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_norm(a, a.post_norm, wred, scratch);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_gemv(a, kDlGateUp, ring, area, red, wred, sx, full, empty, it, ucount, a.gu, false, 0u, 0,
          ok, mk);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  dl_silu(a, wred, scratch);
  mark();
  dl_grid_sync(a.bar, target, ok);
  mark();
  // every CTA has read the epoch (before its first barrier): advance it
  if (tp && blockIdx.x == 0 && tid == 0)
    *reinterpret_cast<volatile uint32_t*>(ctrl) = E + 1u + (a.push_delta ? 1u : 0u);
  const bool push = tp && a.push_delta;
  dl_gemv(a, kDlDown, ring, area, red, wred, sx, full, empty, it, ucount,
          push ? nullptr : a.delta_out, push, E + 2u, static_cast<int>((E + 1u) & 1u), ok, mk);
  mark();
}

}  // namespace lmrs
