// fp8_swap.cuh — FP8 W8A8 linear for 9..64 tokens on tcgen05 (swap-AB).
//
// y[m, n] = bf16(s_x[m] * s_w[n] * sum_k xq[m, k] * wq[n, k] (+ bias[n]))
//
// With few tokens the weight stream is the whole cost, and the register-fed
// GEMV (fp8_gemv_kernel) spends its shared-memory bandwidth re-reading the
// token tile in every warp.  Here the e4m3 weights go from TMA straight into the
// tensor core: a CTA owns 128 output channels (the UMMA M dimension), the tokens
// are the UMMA N dimension (NT = 16, 32 or 64), K advances 128 bytes per stage
// (4 MMAs of K = 32); the fp32 accumulator lives in TMEM.  Clusters of C CTAs
// (a power of two) split K; every CTA sends each channel slice's owner its
// partial sums with 16-byte st.async counted on the owner's mbarrier, and the
// owner applies the scales and bias.
// Warp roles: 0 TMA producer (weights of the first stages before
// griddepcontrol.wait, tokens after), 1 MMA issuer + TMEM owner, 2..5 epilogue
// (TMEM lane quarters).
#pragma once
#include <cooperative_groups.h>
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kFsRows = 128;     // output channels per CTA (UMMA M)
constexpr int kFsBK = 128;       // K bytes per stage
constexpr int kFsThreads = 192;  // producer, MMA, 4 epilogue warps
constexpr int kFsABytes = kFsRows * kFsBK;  // 16 KB
constexpr int kFsMaxCluster = 8;

// NT tokens (UMMA N), ST ring stages; sized for two resident CTAs per SM.
template <int NT, int ST>
struct FsLayout {
  static constexpr int kB = NT * kFsBK;        // token rows x 128 bytes
  static constexpr int kStage = kFsABytes + kB;
  static constexpr int kPitch = NT + 4;        // recv row pitch (floats): float4 reads conflict-free
  static constexpr int kRecv = kFsRows * kPitch * 4;  // [C][cw] rows of NT partials
  static constexpr uint32_t kTmemCols = NT < 32 ? 32 : NT;
  static constexpr int kSmem = 1024 + ST * kStage + kRecv + 256;
  static_assert(kB % 1024 == 0, "128B-swizzled stages are 1024-byte aligned");
  static_assert(2 * kSmem <= 228 * 1024, "two CTAs per SM");
};

template <int NT, int ST>
__global__ void __launch_bounds__(kFsThreads, 2) fp8_swap_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
    __nv_bfloat16* __restrict__ y, const float* __restrict__ sx, const float* __restrict__ sw,
    const __nv_bfloat16* __restrict__ bias, int M, int K, int N) {
  using L = FsLayout<NT, ST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;                                  // [stages][128 rows x 128 B]
  uint8_t* sB = sA + ST * kFsABytes;            // [stages][NT rows x 128 B]
  float* recv = reinterpret_cast<float*>(sB + ST * L::kB);
  uint64_t* full = reinterpret_cast<uint64_t*>(recv + kFsRows * L::kPitch);
  uint64_t* empty = full + ST;
  uint64_t* accfull = empty + ST;
  uint64_t* recv_bar = accfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);

  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int nbase = strip * kFsRows;
  const int cw = kFsRows / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = (K + kFsBK - 1) / kFsBK;
  const int u_lo = static_cast<int>((static_cast<long long>(rank) * units) / C);
  const int u_hi = static_cast<int>((static_cast<long long>(rank + 1) * units) / C);
  const int nk = u_hi - u_lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, kFsRows * NT * 4);  // every peer's slice of this CTA's channels
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_arrive_relaxed();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_x);
      const int pre = nk < ST ? nk : ST;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], L::kStage);
        tma_load_2d(&tm_w, &full[i], sA + i * kFsABytes, (u_lo + i) * kFsBK, nbase);
      }
      pdl_wait();  // the quantised tokens are the previous kernel's output
      for (int i = 0; i < pre; ++i)
        tma_load_2d(&tm_x, &full[i], sB + i * L::kB, (u_lo + i) * kFsBK, 0);
      int s = 0;
      uint32_t ph = 0;
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&empty[s], ph, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[s], L::kStage);
        tma_load_2d(&tm_w, &full[s], sA + s * kFsABytes, (u_lo + i) * kFsBK, nbase);
        tma_load_2d(&tm_x, &full[s], sB + s * L::kB, (u_lo + i) * kFsBK, 0);
        if (++s == ST) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(0, 0, 0, 0, kFsRows, NT);  // e4m3 x e4m3, K-major
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        if (!(ok = mbar_wait(&full[s], ph, kErrWaitFull))) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * kFsABytes);
        const uint32_t b0 = smem_u32(sB + s * L::kB);
#pragma unroll
        for (int kk = 0; kk < kFsBK / 32; ++kk)
          umma_f8(tmem, make_sdesc(a0 + kk * 32, 16, 1024), make_sdesc(b0 + kk * 32, 16, 1024),
                  idesc, (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);
        if (++s == ST) {
          s = 0;
          ph ^= 1;
        }
      }
      umma_commit(accfull);  // also fires (over no MMAs) when this CTA has no K range
    }
  } else {
    // epilogue: TMEM lane quarter q = channels 32q..32q+31; thread = one channel
    const int q = warp & 3;
    const int ch = q * 32 + lane;
    float v[NT];
    if (mbar_wait(accfull, 0, kErrWaitAccum)) {
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
      for (int c = 0; c < NT / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tbase + c * 16, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) v[c * 16 + e] = nk > 0 ? __uint_as_float(r[e]) : 0.f;
      }
    } else {
#pragma unroll
      for (int e = 0; e < NT; ++e) v[e] = 0.f;
    }
    tc_fence_before();
    // partials of channel ch (NT tokens) -> owner r = ch / cw, recv[rank][ch - r*cw][tokens]
    cluster_wait_acquire();
    const int r = ch / cw, cl = ch - r * cw;
    const uint32_t dst =
        mapa_shared(smem_u32(recv + (rank * cw + cl) * L::kPitch), static_cast<uint32_t>(r));
    const uint32_t rbar = mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r));
#pragma unroll
    for (int m4 = 0; m4 < NT; m4 += 4)
      st_async_v4(dst + m4 * 4, make_float4(v[m4], v[m4 + 1], v[m4 + 2], v[m4 + 3]), rbar);
    // owner: thread = (channel c2, 4 tokens); sum the C slices in rank order,
    // scale, bias, store
    const bool ok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
    pdl_wait();
    if (ok) {
      const int M4 = (M + 3) >> 2;
      for (int e = threadIdx.x - 64; e < M4 * cw; e += 128) {
        const int m4 = e / cw, c2 = e - m4 * cw;
        const int n = nbase + rank * cw + c2;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int src = 0; src < C; ++src) {
          const float4 p = *reinterpret_cast<const float4*>(recv + (src * cw + c2) * L::kPitch + 4 * m4);
          acc.x += p.x;
          acc.y += p.y;
          acc.z += p.z;
          acc.w += p.w;
        }
        if (n < N) {
          const float a[4] = {acc.x, acc.y, acc.z, acc.w};
          const float swn = sw[n];
          const float bn = bias != nullptr ? __bfloat162float(bias[n]) : 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int m = 4 * m4 + j;
            if (m < M) {
              float o = __fmul_rn(__fmul_rn(a[j], sx[m]), swn);
              if (bias != nullptr) o = __fadd_rn(o, bn);
              y[static_cast<int64_t>(m) * N + n] = __float2bfloat16_rn(o);
            }
          }
        }
      }
    }
  }
  if (warp < 2) {
    cluster_wait_acquire();  // the non-epilogue warps arrived too; match their wait
    pdl_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace lmrs
