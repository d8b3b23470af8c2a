// allreduce.cuh — one-shot sum all-reduce over NVLink peer memory for the
// row-parallel projections of a tensor-parallel decode step (o and down, a few
// KB to a few hundred KB per call).
//
// Protocol: every rank owns a receive buffer that all ranks map (IPC); it has
// two phases x world slots of 8-byte packets.  A packet carries 4 bytes of data
// (two fp16/bf16 values) and, in its upper half, the flag epoch + 1, written
// by ONE 64-bit store, so a receiver that sees the flag also sees the data: no
// fences, no barrier round trip (the "low-latency" packet scheme of NCCL's LL
// protocol, restated).  Each rank pushes its input into slot `rank` of every
// rank's buffer (itself included), then polls its own buffer until the packets
// of every source carry this call's flag and sums them in rank order, so all
// ranks produce bit-identical results.  Phases alternate with the epoch; a rank
// can only write phase p again two calls later, after every peer has finished
// reading it (each call needs every peer's packets of the call before).  The
// epoch lives in device memory next to the buffer and advances at the end of
// each call (last CTA), so the kernel is CUDA-graph replayable.
// Every wait is bounded: on expiry the kernel sets kErrWaitPeer, stops waiting
// for the rest of the call and writes NaN wherever a source's packet was
// missing, so a lost peer cannot pass for a valid sum downstream.
#pragma once
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kArMaxRanks = 8;
constexpr int kArThreads = 256;

struct ArPeers {
  uint64_t* buf[kArMaxRanks];  // every rank's receive packets (device pointers, mapped)
};

// receive-buffer layout: [64-byte control: epoch, finished-CTA count][2][world][cap] packets
__device__ __forceinline__ void st_sys_b64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_b64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The same load without volatile / memory clobber, so that several of them can
// be in flight together: only for a first look, never inside a polling loop
// (the compiler may merge repeated calls on the same address).
__device__ __forceinline__ uint64_t ld_sys_b64_once(const uint64_t* p) {
  uint64_t v;
  asm("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kArThreads) allreduce_ll_kernel(T* out,
                                                                  const T* in,  // may alias out
                                                                  int n2, int rank, int world,
                                                                  ArPeers peers, int cap) {
  pdl_wait();  // the input is the previous kernel's output
  pdl_trigger();
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(peers.buf[rank]) - 16;  // 64-byte header
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ctrl);
  const uint64_t flag = static_cast<uint64_t>(epoch + 1u) << 32;
  const int phase = static_cast<int>(epoch & 1u);
  const uint32_t* in32 = reinterpret_cast<const uint32_t*>(in);
  const int stride = gridDim.x * blockDim.x;
  const int i0 = blockIdx.x * blockDim.x + threadIdx.x;

  // push: this rank's packets into slot `rank` of every rank's buffer
  for (int i = i0; i < n2; i += stride) {
    const uint64_t pkt = flag | in32[i];
    for (int p = 0; p < world; ++p)
      st_sys_b64(peers.buf[p] + (static_cast<int64_t>(phase) * world + rank) * cap + i, pkt);
  }

  // receive: wait for each source's packet, sum in rank order
  const uint64_t* own = peers.buf[rank] + static_cast<int64_t>(phase) * world * cap;
  bool ok = true;
  for (int i = i0; i < n2; i += stride) {
    float a0 = 0.f, a1 = 0.f;
    for (int s = 0; s < world; ++s) {
      const uint64_t* src = own + static_cast<int64_t>(s) * cap + i;
      uint64_t pkt = ld_sys_b64(src);
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
      const uint32_t v = static_cast<uint32_t>(pkt);
      T pair[2];
      *reinterpret_cast<uint32_t*>(pair) = v;
      a0 += static_cast<float>(pair[0]);
      a1 += static_cast<float>(pair[1]);
    }
    T res[2] = {T(a0), T(a1)};
    reinterpret_cast<uint32_t*>(out)[i] = *reinterpret_cast<uint32_t*>(res);
  }

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

// Two-stage form for large messages at many ranks (the one-shot kernel pushes
// world x n packets per rank, this one about 2n): the packets are cut into
// `world` slices, slice r owned by rank r.
//   1. reduce-scatter: every rank pushes its packets of slice r into slot
//      `rank` of rank r's buffer (the one-shot layout, only slice r's range);
//   2. the owner polls its slice's packets from every source, sums them in rank
//      order (the one-shot kernel's arithmetic, so the result is the same),
//      writes its output and pushes each rounded pair as an all-gather packet
//      into slot `rank` of every other rank's buffer at the same index: in
//      rank q's buffer, slot r at indices of slice r is never written by the
//      reduce-scatter (rank r sends there only slice q), so the two never mix;
//   3. every rank polls the other slices' all-gather packets and writes them.
// Same flag / epoch / phase protocol and bounded waits as the one-shot kernel;
// no CTA waits on another CTA of its own grid.
template <typename T>
__global__ void __launch_bounds__(kArThreads) allreduce_2stage_kernel(T* out, const T* in, int n2,
                                                                      int rank, int world,
                                                                      ArPeers peers, int cap) {
  pdl_wait();  // the input is the previous kernel's output
  pdl_trigger();
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(peers.buf[rank]) - 16;  // 64-byte header
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ctrl);
  const uint64_t flag = static_cast<uint64_t>(epoch + 1u) << 32;
  const int phase = static_cast<int>(epoch & 1u);
  const uint32_t* in32 = reinterpret_cast<const uint32_t*>(in);
  uint32_t* out32 = reinterpret_cast<uint32_t*>(out);
  const int stride = gridDim.x * blockDim.x;
  const int i0 = blockIdx.x * blockDim.x + threadIdx.x;
  const int per = (n2 + world - 1) / world;  // packets per slice
  auto slot = [&](int dst, int src) {
    return peers.buf[dst] + (static_cast<int64_t>(phase) * world + src) * cap;
  };
  auto wait_pkt = [&](const uint64_t* src, bool& ok) -> uint64_t {
    uint64_t pkt = ld_sys_b64(src);
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
    return pkt;
  };

  // 1. reduce-scatter: packets of slice r to rank r (its own slice too)
  for (int k = i0; k < n2; k += stride) {
    const int r = k / per;
    st_sys_b64(slot(r, rank) + k, flag | in32[k]);
  }
  // 2. own slice: rank-order sum, output, all-gather packets to the others
  bool ok = true;
  const int lo = rank * per, hi = min(n2, lo + per);
  const uint64_t* own = peers.buf[rank] + static_cast<int64_t>(phase) * world * cap;
  for (int k = lo + i0; k < hi; k += stride) {
    float a0 = 0.f, a1 = 0.f;
    for (int s = 0; s < world; ++s) {
      const uint64_t pkt = wait_pkt(own + static_cast<int64_t>(s) * cap + k, ok);
      if ((pkt & 0xFFFFFFFF00000000ull) != flag) {  // gave up on this source
        a0 = a1 = __int_as_float(0x7fc00000);
        continue;
      }
      const uint32_t v = static_cast<uint32_t>(pkt);
      T pair[2];
      *reinterpret_cast<uint32_t*>(pair) = v;
      a0 += static_cast<float>(pair[0]);
      a1 += static_cast<float>(pair[1]);
    }
    T res[2] = {T(a0), T(a1)};
    const uint32_t rv = *reinterpret_cast<uint32_t*>(res);
    out32[k] = rv;
    for (int q = 0; q < world; ++q)
      if (q != rank) st_sys_b64(slot(q, rank) + k, flag | rv);
  }
  // 3. the other slices, from their owners
  for (int k = i0; k < n2; k += stride) {
    const int r = k / per;
    if (r == rank) continue;
    const uint64_t pkt = wait_pkt(own + static_cast<int64_t>(r) * cap + k, ok);
    out32[k] = (pkt & 0xFFFFFFFF00000000ull) == flag ? static_cast<uint32_t>(pkt) : 0x7fc07fc0u;
  }

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
