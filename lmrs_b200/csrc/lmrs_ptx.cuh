// lmrs_ptx.cuh — sm_100a device primitives used by the quantized-linear kernels:
// bounded mbarrier waits, TMA tile loads, tcgen05 (TMEM alloc / MMA / commit /
// load), UMMA shared-memory and instruction descriptors, and the magic-number
// int4 -> fp16 conversion.  Everything is hand-written inline PTX; no CUTLASS.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace lmrs {

// ---------------------------------------------------------------- error word
// One word per device (module-scope __device__ variable).  A kernel whose
// bounded wait expires ORs a site bit in here and unwinds instead of hanging.
// Host side: lmrs_read_device_error().
enum : uint32_t {
  kErrWaitFull = 1u << 0,      // consumer waiting for a TMA stage
  kErrWaitEmpty = 1u << 1,     // producer waiting for a free stage
  kErrWaitAccum = 1u << 2,     // epilogue waiting for the accumulator
  kErrWaitDequant = 1u << 3,   // MMA waiting for the dequantised B stage
  kErrWaitCluster = 1u << 4,   // cluster reduction waiting for peers
  kErrWaitPeer = 1u << 5,      // all-reduce waiting for another GPU's packets
  kErrWaitGrid = 1u << 6,      // persistent kernel waiting at a grid-wide barrier
};

__device__ uint32_t g_device_error;

// ~2 s at 1.9 GHz: far above any legitimate wait in these kernels.
constexpr long long kWaitLimitCycles = 4000000000LL;
// The limit every bounded wait uses, per device; kWaitLimitCycles unless a
// host lowers it (lmrs_set_tuning "wait_limit_kcycles", e.g. to make a test's
// wait on an arrival that never comes give up within a millisecond).  A wait
// reads it only once it has lasted kWaitCheckCycles (~0.5 ms): a global load
// on every wait that misses its first try put L2 latency on the critical path
// of the GEMM pipelines.  Limits below kWaitCheckCycles act as kWaitCheckCycles.
__device__ long long g_wait_limit_cycles = kWaitLimitCycles;
constexpr long long kWaitCheckCycles = 1LL << 20;

// True once a wait that started at t0 has outlived the device's limit.
__device__ __forceinline__ bool wait_expired(long long t0, long long& limit) {
  const long long el = clock64() - t0;
  if (el < kWaitCheckCycles) return false;
  if (limit < 0) limit = *static_cast<volatile long long*>(&g_wait_limit_cycles);
  return el > limit;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// try_wait with a suspend-time hint: a waiting warp sleeps (up to the hint, in
// ns) until the phase completes instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Bounded: after
// g_wait_limit_cycles it records `site` in the device error word and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  long long limit = -1;
  while (!mbar_try_wait(bar, parity)) {
    if (wait_expired(t0, limit)) {
      atomicOr(&g_device_error, site);
      return false;
    }
  }
  return true;
}

// The same wait for a thread on a critical path that usually finds the phase
// complete: a non-blocking test_wait first (measured ~90 cycles against ~130
// for a try_wait on a completed phase), the bounded try_wait loop otherwise.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity, uint32_t site) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0 || mbar_wait(bar, parity, site);
}

// ----------------------------------------------------------------- proxies
// Generic-proxy shared-memory writes -> visible to the async proxy (UMMA reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled load global -> shared, completion counted on `bar` (bytes).
// c0 is the innermost (contiguous) coordinate.  No multicast, ever.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* m, uint64_t* bar, void* dst,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Same, with an L2 eviction-priority hint (createpolicy result).
__device__ __forceinline__ void tma_load_2d_hint(const CUtensorMap* m, uint64_t* bar, void* dst,
                                                 int32_t c0, int32_t c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (fp16/bf16 in, fp32 acc).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f8f6f4 (e4m3/e5m2/... in, fp32 acc), K = 32 per instruction.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with the A operand read from tensor memory (lane = row of A, each 32-bit
// column holds two consecutive K elements); B from a shared-memory descriptor.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns from registers: thread t of the
// warp writes TMEM lane (base_lane + t), columns [col, col+16).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Same, 32 consecutive columns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 16 lanes x 128 bits, four repetitions along the columns: register 2j goes to
// TMEM lane (base_lane + t/4), column (col + 4j + t%4); register 2j+1 to lane
// (base_lane + 8 + t/4), the same column (t = thread of the warp).
__device__ __forceinline__ void tmem_st16x128b_x4(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns: thread t of the warp receives
// TMEM lane (base_lane + t), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 bits, 4 consecutive columns.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// ------------------------------------------------- 2-SM (CTA pair) variants
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier anywhere in the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
          cluster_addr),
      "r"(bytes)
      : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_cg2(const CUtensorMap* m, uint32_t bar_cluster,
                                                void* dst, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_cg2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_cg2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (M=256 across the pair) (+)= A * B, both CTAs' shared memory at the same offsets.
__device__ __forceinline__ void umma_f16_cg2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f8f6f4 on the pair (M = 256 across the two CTAs, K = 32 per instruction).
__device__ __forceinline__ void umma_f8_cg2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at this offset in every CTA of `cta_mask` when the
// pair's previously issued MMAs complete.
__device__ __forceinline__ void umma_commit_cg2_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Split cluster barrier: arrive early (after mbarrier init + fence_mbar_init),
// wait just before the first access to a peer's shared memory.
// (Non-.aligned forms: callers may reach them from divergent code.)
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ float4 ld_cluster_v4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}

// Asynchronous 16-byte store into a peer CTA's shared memory whose completion
// is counted (in bytes) on an mbarrier in that CTA: no release fence needed,
// the receiver's wait on the mbarrier makes the data visible.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, float4 v, uint32_t cluster_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
      ::"r"(cluster_addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cluster_bar)
      : "memory");
}

// Bounded wait that also acquires at cluster scope (data written into this
// CTA's shared memory by peer CTAs before their release-arrive).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t site) {
  const long long t0 = clock64();
  long long limit = -1;
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    if (ok) return true;
    if (wait_expired(t0, limit)) {
      atomicOr(&g_device_error, site);
      return false;
    }
  }
}

// ------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialisation may start while
// the previous kernel in the stream is still running.  pdl_trigger lets the
// next kernel start launching; pdl_wait blocks until the previous kernel has
// completed and its writes are visible.  Both are no-ops without the launch
// attribute.  Every kernel here reads its activations and writes any global
// memory only after pdl_wait; weights (never written by a predecessor) may be
// prefetched before it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor (sm_100 format):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1, [49,52) base offset,
//   [52] lbo mode, [61,64) layout (2 = 128-byte swizzle).
// K-major SW128 tile (rows x 128 B, 8-row atoms of 1024 B): SBO = 1024, LBO unused.
// MN-major SW128 tile: 64-element (128 B) MN blocks at stride LBO, 8-row K groups
// at stride SBO.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // version (sm_100)
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, dense, fp32 accumulate:
//   [4,6) c format (1 = f32), [7,10) a format, [10,13) b format,
//   [15] a major (0 = K, 1 = MN), [16] b major, [17,23) N >> 3, [24,29) M >> 4.
// kind::f16: format 0 = f16, 1 = bf16.  kind::f8f6f4: 0 = e4m3, 1 = e5m2.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t a_fmt, uint32_t b_fmt,
                                                  uint32_t a_mn_major, uint32_t b_mn_major,
                                                  uint32_t M, uint32_t N) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ldmatrix, four 8x8 b16 matrices; lanes 8j .. 8j+7 give the row addresses of
// matrix j.  Plain: thread t gets row t/4, columns 2(t%4), 2(t%4)+1 of each;
// .trans: column t/4 of rows 2(t%4) (low half) and 2(t%4)+1 (high half).
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// ------------------------------------------------------------- int4 dequant
// AWQ packs column 8j+ORDER[i] into nibble i with ORDER = {0,2,4,6,1,3,5,7}, so
// (w >> 4t) & 0x000F000F holds columns (2t, 2t+1) in its two 16-bit halves.
// OR-ing 0x6400 (fp16 1024.0, ulp 1) makes each half exactly 1024 + nibble.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));
  return r;  // (a & mask) | magic
}

// Four half2 = (1024 + v_c, 1024 + v_{c+1}) for columns (0,1),(2,3),(4,5),(6,7).
__device__ __forceinline__ void awq_word_to_h2_biased(uint32_t w, uint32_t (&h)[4]) {
  h[0] = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  h[1] = lop3_and_or(w >> 4, 0x000F000Fu, 0x64006400u);
  h[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x64006400u);
  h[3] = lop3_and_or(w >> 12, 0x000F000Fu, 0x64006400u);
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) {
  return *reinterpret_cast<__half2*>(&v);
}

// fp16_rne((q - z) * s): (1024+q) - (1024+z) is exact, the fp16 multiply rounds once.
__device__ __forceinline__ uint32_t dq_h2(uint32_t qb, uint32_t zb, uint32_t s) {
  return h2_as_u32(__hmul2(__hsub2(u32_as_h2(qb), u32_as_h2(zb)), u32_as_h2(s)));
}

// ------------------------------------------- activation types of the AWQ path
// Every AWQ kernel runs with fp16 (LMRS_DTYPE_F16) or bf16 (LMRS_DTYPE_BF16)
// activations; x, y, bias and the dequantised weight share that type, the
// scales stay fp16 as stored.  The dequantised weight is always the exact
// product (q - z) * s rounded once to the activation type.  What differs:
//   * the magic-number bias: fp16 has 10 mantissa bits, so a nibble in bits
//     0-3 of a half gives 1024 + q (0x6400) and one in bits 4-7 gives 64 + q
//     (0x5400, ulp 1/16); bf16 has 7, so every nibble is first shifted to bits
//     0-3 and gives 128 + q (0x4300, ulp 1);
//   * the product: the fp16 multiply of (q - z) (exact) by s rounds once.  A
//     bf16 multiply cannot take the fp16 scale, so s is split into
//     s_hi = bf16_rne(s) and s_lo = s - s_hi (at most 3 significant bits,
//     exact in bf16); d * s_lo is exact (|d| <= 15), and one
//     fma.rn.bf16x2(d, s_hi, d * s_lo) rounds d * s once;
//   * the UMMA / mma.sync operand format.
template <typename T>
struct Act;
template <>
struct Act<__half> {
  static constexpr uint32_t kUmmaFmt = 0;          // kind::f16 operand format: f16
  static constexpr uint32_t kOne2 = 0x3C003C00u;   // (1, 1)
  static constexpr CUtensorMapDataType kTma = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  static constexpr float kMaxFinite = 65504.f;
  __device__ __forceinline__ static float to_float(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_float(float v) { return __float2half_rn(v); }
  __device__ __forceinline__ static float2 unpack2(uint32_t v) {
    return __half22float2(u32_as_h2(v));
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    return h2_as_u32(__floats2half2_rn(a, b));
  }
};
template <>
struct Act<__nv_bfloat16> {
  static constexpr uint32_t kUmmaFmt = 1;          // kind::f16 operand format: bf16
  static constexpr uint32_t kOne2 = 0x3F803F80u;
  static constexpr CUtensorMapDataType kTma = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  static constexpr float kMaxFinite = 3.38953139e38f;
  __device__ __forceinline__ static float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static float2 unpack2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float v) {
    return __float2bfloat16_rn(v);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Biased pair (B + q_lo, B + q_hi) of nibble j (bits 4j .. 4j+3) of each
// 16-bit half of v; B = awq_nib_bias<T>(j).
template <typename T>
__device__ __forceinline__ uint32_t awq_nib_pair(uint32_t v, int j) {
  if constexpr (Act<T>::kUmmaFmt == 0) {
    const uint32_t u = (j & 2) ? v >> 8 : v;
    return (j & 1) ? lop3_and_or(u, 0x00F000F0u, 0x54005400u)
                   : lop3_and_or(u, 0x000F000Fu, 0x64006400u);
  } else {
    return lop3_and_or(v >> (4 * j), 0x000F000Fu, 0x43004300u);
  }
}
template <typename T>
__host__ __device__ constexpr float awq_nib_bias(int j) {
  return Act<T>::kUmmaFmt == 0 ? ((j & 1) ? 64.f : 1024.f) : 128.f;
}
// The zero point z (0..15) biased like nibble j, in both halves.
template <typename T>
__device__ __forceinline__ uint32_t awq_zero_pair(uint32_t z, int j) {
  if constexpr (Act<T>::kUmmaFmt == 0)
    return ((j & 1) ? (0x5400u | (z << 4)) : (0x6400u | z)) * 0x00010001u;
  else
    return (0x4300u | z) * 0x00010001u;
}

// Four biased pairs for columns (0,1),(2,3),(4,5),(6,7) of one packed word
// (every nibble shifted to bits 0-3: bias 1024 for fp16, 128 for bf16).
template <typename T>
__device__ __forceinline__ void awq_word_biased(uint32_t w, uint32_t (&h)[4]) {
  constexpr uint32_t magic = Act<T>::kUmmaFmt == 0 ? 0x64006400u : 0x43004300u;
  h[0] = lop3_and_or(w, 0x000F000Fu, magic);
  h[1] = lop3_and_or(w >> 4, 0x000F000Fu, magic);
  h[2] = lop3_and_or(w >> 8, 0x000F000Fu, magic);
  h[3] = lop3_and_or(w >> 12, 0x000F000Fu, magic);
}

// The scale operand of a pair of channels (two fp16 scales in s16x2): fp16
// keeps the pair as is; bf16 keeps (s_hi pair, s_lo pair).
struct AwqScale2 {
  uint32_t hi, lo;
};
template <typename T>
__device__ __forceinline__ AwqScale2 awq_scale2(uint32_t s16x2) {
  if constexpr (Act<T>::kUmmaFmt == 0) {
    return {s16x2, 0u};
  } else {
    const float2 f = __half22float2(u32_as_h2(s16x2));
    const __nv_bfloat162 hi = __floats2bfloat162_rn(f.x, f.y);
    const float2 fh = __bfloat1622float2(hi);
    // s - s_hi is exact in fp32; an infinite scale keeps s_lo = 0 so that
    // d * s stays +-inf (NaN for d = 0) as in the exact product
    const float lx = isinf(fh.x) ? 0.f : f.x - fh.x;
    const float ly = isinf(fh.y) ? 0.f : f.y - fh.y;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(lx, ly);
    return {*reinterpret_cast<const uint32_t*>(&hi), *reinterpret_cast<const uint32_t*>(&lo)};
  }
}

// T_rne((q - z) * s) for a pair from biased q and z pairs.
template <typename T>
__device__ __forceinline__ uint32_t awq_dq(uint32_t qb, uint32_t zb, AwqScale2 s) {
  if constexpr (Act<T>::kUmmaFmt == 0) {
    return dq_h2(qb, zb, s.hi);
  } else {
    uint32_t d, t, w;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(qb), "r"(zb));      // exact
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(d), "r"(s.lo));     // exact
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(w) : "r"(d), "r"(s.hi), "r"(t));
    return w;
  }
}

}  // namespace lmrs
