// allreduce_norm.cuh — the row-parallel projection's all-reduce fused with the
// residual add and RMSNorm that follow it in a tensor-parallel decode step:
//
//   delta    = sum over ranks of part (fp32, rank order, rounded once to T:
//              bit-identical to allreduce_ll_kernel's result)
//   residual = T(residual + delta)                    (in place, as rmsnorm_kernel)
//   out      = T(residual * rsqrt(mean(residual^2) + eps) * w)
//   FP8 form: the e4m3 bytes and per-row scale of that rounded output instead
//
// One launch instead of two (all-reduce, then norm): at batch 1 a decode step's
// small kernels each cost a launch's latency on the dependency chain whatever
// their size, and a tensor-parallel layer has two of these pairs.
//
// Layout: a thread-block cluster of C CTAs per row (C = ceil(H / 1024) up to 8),
// CTA r of a cluster owning columns [r * VPT * 1024, (r + 1) * VPT * 1024),
// one packet (two columns) per thread and step: as many threads push and poll
// as the all-reduce kernel uses.  The clusters walk the rows (grid-stride);
// the grid is sized so that every CTA is resident at once, because the CTAs of
// all ranks wait on one another's packets.  Every cluster first pushes the
// packets of all its rows to every rank (the all-reduce's 8-byte data + epoch
// packets, same buffers, same epoch / phase protocol), then takes its rows one
// by one: poll its own buffer until each source's packets of the slice carry
// this call's flag, sum in rank order, update the residual, and reduce the
// row's sum of squares (and, FP8, its maximum) over the cluster through
// distributed shared memory: each CTA stores its partial into slot[rank] of
// every CTA of the cluster, and after a cluster barrier every CTA adds the C
// partials in rank order (the same total in all of them).  Bounded waits as in
// allreduce_ll_kernel: a missing source's packets count as NaN and the kernel
// sets kErrWaitPeer.
#pragma once
#include <cooperative_groups.h>
#include "allreduce.cuh"
#include "decode_ops.cuh"

namespace lmrs {

constexpr int kArnThreads = 512;
constexpr int kArnMaxCluster = 8;
constexpr int kArnMaxVecs = 4;
constexpr int kArnCols = kArnThreads * 2;  // columns of one step of a CTA (one packet per thread)

// Two rounded activations -> two e4m3 bytes with the row scale s (the pairing
// of e4m3x8, so the bytes equal fp8_quant_rows_kernel's).
__device__ __forceinline__ uint16_t e4m3x2(float a, float b, float s) {
  if (s == 0.f) return 0;
  const float2 pr = make_float2(__fdiv_rn(a, s), __fdiv_rn(b, s));
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(pr, __NV_SATFINITE, __NV_E4M3));
}


template <typename T, bool FP8, int VPT>
__global__ void __launch_bounds__(kArnThreads) allreduce_rmsnorm_kernel(
    T* __restrict__ out, uint8_t* __restrict__ qout, float* __restrict__ qscale,
    T* __restrict__ resid, const T* __restrict__ part, const T* __restrict__ w, int rows, int H,
    float eps, int rank, int world, ArPeers peers, int cap) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int cr = static_cast<int>(cluster.block_rank());
  const int clu = blockIdx.x / C, nclu = gridDim.x / C;
  __shared__ float red[32];
  __shared__ float slot[2][kArnMaxCluster];
  cluster_arrive_relaxed();  // peers' shared memory is used only after the matching wait
  const int c0 = cr * VPT * kArnCols + threadIdx.x * 2;  // column of this thread's pair, step 0
  // the norm weight is constant: read before the previous kernel has finished
  uint32_t wv[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v)
    wv[v] = c0 + v * kArnCols < H ? __ldg(reinterpret_cast<const uint32_t*>(w + c0 + v * kArnCols)) : 0u;
  pdl_wait();  // the partial sums are the previous kernel's output
  pdl_trigger();
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(peers.buf[rank]) - 16;  // 64-byte header
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ctrl);
  const uint64_t flag = static_cast<uint64_t>(epoch + 1u) << 32;
  const int phase = static_cast<int>(epoch & 1u);

  // ---- push: this rank's packets of every row of the cluster, to every rank
  for (int row = clu; row < rows; row += nclu) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int c = c0 + v * kArnCols;
      if (c >= H) continue;
      const int64_t e = static_cast<int64_t>(row) * H + c;
      const uint64_t pkt = flag | *reinterpret_cast<const uint32_t*>(part + e);
      for (int p = 0; p < world; ++p)
        st_sys_b64(peers.buf[p] + (static_cast<int64_t>(phase) * world + rank) * cap + (e >> 1), pkt);
    }
  }

  // ---- per row: receive, residual, norm
  const uint64_t* own = peers.buf[rank] + static_cast<int64_t>(phase) * world * cap;
  bool ok = true;
  bool first = true;
  for (int row = clu; row < rows; row += nclu) {
    const int64_t rb = static_cast<int64_t>(row) * H;
    // the residual pairs and every source's packets, requested at once
    uint32_t rv[VPT];
    uint64_t pk[VPT][kArMaxRanks];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int c = c0 + v * kArnCols;
      rv[v] = c < H ? *reinterpret_cast<const uint32_t*>(resid + rb + c) : 0u;
#pragma unroll
      for (int s = 0; s < kArMaxRanks; ++s)
        if (c < H && s < world) pk[v][s] = ld_sys_b64_once(own + static_cast<int64_t>(s) * cap + ((rb + c) >> 1));
    }
    float x[VPT][2];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int c = c0 + v * kArnCols;
      if (c >= H) continue;
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int s = 0; s < kArMaxRanks; ++s) {
        if (s >= world) break;
        const uint64_t* src = own + static_cast<int64_t>(s) * cap + ((rb + c) >> 1);
        uint64_t pkt = pk[v][s];
        if ((pkt & 0xFFFFFFFF00000000ull) != flag) {
          const long long t0 = clock64();
          long long limit = -1;
          while (ok && ((pkt = ld_sys_b64(src)) & 0xFFFFFFFF00000000ull) != flag) {
            if (wait_expired(t0, limit)) {
              atomicOr(&g_device_error, kErrWaitPeer);
              ok = false;
            }
          }
        }
        if ((pkt & 0xFFFFFFFF00000000ull) != flag) {  // gave up on this source
          a0 = a1 = __int_as_float(0x7fc00000);
          continue;
        }
        const float2 f = unpack2<T>(static_cast<uint32_t>(pkt));
        a0 += f.x;
        a1 += f.y;
      }
      // the all-reduce's rounding, then the residual update as rmsnorm_kernel's
      const float2 d = unpack2<T>(pack2<T>(a0, a1));
      const float2 r = unpack2<T>(rv[v]);
      const uint32_t nv = pack2<T>(r.x + d.x, r.y + d.y);
      const float2 xn = unpack2<T>(nv);
      x[v][0] = xn.x;
      x[v][1] = xn.y;
      ss += xn.x * xn.x + xn.y * xn.y;
      *reinterpret_cast<uint32_t*>(resid + rb + c) = nv;  // the updated residual stream
    }
    // row sum of squares over the cluster
    const float local = block_sum(ss, red);
    if (first) {
      cluster_wait_acquire();  // every CTA of the cluster is running
      first = false;
    } else {
      cluster_sync_all();  // the previous row's slots have been read everywhere
    }
    if (threadIdx.x < C)
      st_cluster_f32(mapa_shared(smem_u32(&slot[0][cr]), static_cast<uint32_t>(threadIdx.x)), local);
    cluster_sync_all();
    float tot = 0.f;
    for (int q = 0; q < C; ++q) tot += slot[0][q];
    const float inv = rsqrtf(tot / H + eps);
    float amax = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int c = c0 + v * kArnCols;
      if (c >= H) continue;
      const float2 wf = unpack2<T>(wv[v]);
      const uint32_t o = pack2<T>(x[v][0] * inv * wf.x, x[v][1] * inv * wf.y);
      const float2 of = unpack2<T>(o);
      x[v][0] = of.x;
      x[v][1] = of.y;
      amax = fmaxf(amax, fmaxf(fabsf(of.x), fabsf(of.y)));
      if (!FP8) *reinterpret_cast<uint32_t*>(out + rb + c) = o;
    }
    if (FP8) {
      const float lmax = block_max(amax, red);
      if (threadIdx.x < C)
        st_cluster_f32(mapa_shared(smem_u32(&slot[1][cr]), static_cast<uint32_t>(threadIdx.x)), lmax);
      cluster_sync_all();
      float rmax = slot[1][0];
      for (int q = 1; q < C; ++q) rmax = fmaxf(rmax, slot[1][q]);
      const float sc = __fdiv_rn(rmax, 448.0f);
      if (cr == 0 && threadIdx.x == 0) qscale[row] = sc;
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int c = c0 + v * kArnCols;
        if (c < H) *reinterpret_cast<uint16_t*>(qout + rb + c) = e4m3x2(x[v][0], x[v][1], sc);
      }
    }
  }
  // every store into a peer's slots came before that row's exchange barrier, so
  // a CTA may leave now; a cluster without rows still matches its arrive
  if (first) cluster_wait_acquire();

  // advance the epoch once every CTA is done with this call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctrl + 1, 1u) == gridDim.x - 1) {
      ctrl[1] = 0u;
      *reinterpret_cast<volatile uint32_t*>(ctrl) = epoch + 1u;
    }
  }
}

}  // namespace lmrs
