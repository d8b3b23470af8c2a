// comm_capi.cuh — the C-ABI of include/lmrs_comm.h (included at the end of
// lmrs_capi.cu, one translation unit with the other entry points).
#pragma once
#include "allreduce.cuh"
#include "lmrs_comm.h"

namespace {

constexpr size_t kArHeader = 64;

size_t ar_cap(size_t max_elems) { return (max_elems + 1) / 2; }

template <typename T>
int allreduce_launch(void* out, const void* in, size_t n, int rank, int world,
                     void* const* buffers, size_t max_elems, cudaStream_t st, int dev) {
  lmrs::ArPeers peers = {};
  for (int r = 0; r < world; ++r)
    peers.buf[r] = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(buffers[r]) + kArHeader);
  const int n2 = static_cast<int>(n / 2);
  int grid = (n2 + lmrs::kArThreads - 1) / lmrs::kArThreads;
  // every CTA resident at once: the CTAs of all ranks wait on one another
  if (grid > sm_count(dev)) grid = sm_count(dev);
  if (grid < 1) grid = 1;
  int rc = launch_ex(lmrs::allreduce_ll_kernel<T>, grid, 0, lmrs::kArThreads, 0, st,
                     static_cast<T*>(out), static_cast<const T*>(in), n2, rank, world, peers,
                     static_cast<int>(ar_cap(max_elems)));
  return rc ? rc : after_launch();
}

}  // namespace

extern "C" {

LMRS_API size_t lmrs_allreduce_buffer_bytes(int world, size_t max_elems) {
  if (world <= 0 || world > lmrs::kArMaxRanks) return 0;
  return kArHeader + 2 * static_cast<size_t>(world) * ar_cap(max_elems) * sizeof(uint64_t);
}

LMRS_API int lmrs_comm_alloc(void** ptr_out, size_t bytes) {
  if (!ptr_out) return LMRS_ERR_NULL;
  if (bytes == 0) return LMRS_ERR_SHAPE;
  int rc = check_device(nullptr);
  if (rc) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return record(e);
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return record(e);
  }
  *ptr_out = p;
  return LMRS_OK;
}

LMRS_API int lmrs_comm_free(void* ptr) {
  if (!ptr) return LMRS_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? LMRS_OK : record(e);
}

LMRS_API int lmrs_ipc_get_handle(void* ptr, void* handle_out, size_t handle_bytes) {
  if (!ptr || !handle_out) return LMRS_ERR_NULL;
  if (handle_bytes < sizeof(cudaIpcMemHandle_t)) return LMRS_ERR_SHAPE;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return record(e);
  memcpy(handle_out, &h, sizeof(h));
  return LMRS_OK;
}

LMRS_API int lmrs_ipc_open(const void* handle, void** ptr_out) {
  if (!handle || !ptr_out) return LMRS_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? LMRS_OK : record(e);
}

LMRS_API int lmrs_ipc_close(void* ptr) {
  if (!ptr) return LMRS_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? LMRS_OK : record(e);
}

LMRS_API int lmrs_allreduce_sum(void* out, const void* in, size_t n, int dtype, int rank,
                                int world, void* const* buffers, size_t max_elems,
                                lmrs_stream_t stream) {
  if (dtype != LMRS_DTYPE_BF16 && dtype != LMRS_DTYPE_F16) return LMRS_ERR_DTYPE;
  if (world <= 0 || world > lmrs::kArMaxRanks || rank < 0 || rank >= world || n % 2 ||
      n > max_elems || max_elems / 2 > static_cast<size_t>(INT32_MAX))
    return LMRS_ERR_SHAPE;
  if (n == 0) return LMRS_OK;
  if (!out || !in || !buffers) return LMRS_ERR_NULL;
  for (int r = 0; r < world; ++r)
    if (!buffers[r]) return LMRS_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(out) & 3u) || (reinterpret_cast<uintptr_t>(in) & 3u))
    return LMRS_ERR_ALIGN;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? allreduce_launch<__nv_bfloat16>(out, in, n, rank, world, buffers, max_elems, st, dev)
             : allreduce_launch<__half>(out, in, n, rank, world, buffers, max_elems, st, dev);
}

}  // extern "C"
