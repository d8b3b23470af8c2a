// comm_capi.cuh — the C-ABI of include/lmrs_comm.h (included at the end of
// lmrs_capi.cu, one translation unit with the other entry points).
#pragma once
#include "allreduce.cuh"
#include "allreduce_norm.cuh"
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
  const bool two = world >= g_tune.ar_two_stage_min_world &&
                   static_cast<long long>(n) >= g_tune.ar_two_stage_min_elems;
  int rc = launch_ex(two ? lmrs::allreduce_2stage_kernel<T> : lmrs::allreduce_ll_kernel<T>, grid,
                     0, lmrs::kArThreads, 0, st, static_cast<T*>(out), static_cast<const T*>(in),
                     n2, rank, world, peers, static_cast<int>(ar_cap(max_elems)));
  return rc ? rc : after_launch();
}

// Fused all-reduce + residual add + RMSNorm: a cluster of C CTAs per row
// (1024 columns per CTA and step), the clusters walking the rows; no more
// clusters than the device holds at once, so that every CTA of every rank is
// resident together.
template <typename T, bool FP8>
int allreduce_norm_launch(void* out, uint8_t* q_out, float* scale_out, void* residual,
                          const void* partial, const void* weight, int rows, int H, float eps,
                          int rank, int world, void* const* buffers, size_t max_elems,
                          cudaStream_t st, int dev) {
  lmrs::ArPeers peers = {};
  for (int r = 0; r < world; ++r)
    peers.buf[r] = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(buffers[r]) + kArHeader);
  int C = (H + lmrs::kArnCols - 1) / lmrs::kArnCols;
  if (C > lmrs::kArnMaxCluster) C = lmrs::kArnMaxCluster;
  const int vpt = (H + C * lmrs::kArnCols - 1) / (C * lmrs::kArnCols);
  const int cap = static_cast<int>(ar_cap(max_elems));
  auto go = [&](auto kern) -> int {
    // as many clusters as the device holds at once (the CTAs of all ranks wait
    // on one another's packets, so none may wait for a slot), at most one per row
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C, 1, 1);
    cfg.blockDim = dim3(lmrs::kArnThreads, 1, 1);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = C;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int resident = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&resident, kern, &cfg);
    if (e != cudaSuccess) return record(e);
    if (resident < 1) return static_cast<int>(LMRS_ERR_SHAPE);
    const int nclu = rows < resident ? rows : resident;
    return launch_ex(kern, nclu * C, C, lmrs::kArnThreads, 0, st, static_cast<T*>(out), q_out,
                     scale_out, static_cast<T*>(residual), static_cast<const T*>(partial),
                     static_cast<const T*>(weight), rows, H, eps, rank, world, peers, cap);
  };
  int rc = vpt == 1   ? go(lmrs::allreduce_rmsnorm_kernel<T, FP8, 1>)
           : vpt == 2 ? go(lmrs::allreduce_rmsnorm_kernel<T, FP8, 2>)
           : vpt == 3 ? go(lmrs::allreduce_rmsnorm_kernel<T, FP8, 3>)
                      : go(lmrs::allreduce_rmsnorm_kernel<T, FP8, 4>);
  return rc ? rc : after_launch();
}

int allreduce_norm_check(const void* outp, void* residual, const void* partial,
                         const void* weight, int rows, int H, int dtype, int rank, int world,
                         void* const* buffers, size_t max_elems) {
  if (dtype != LMRS_DTYPE_BF16 && dtype != LMRS_DTYPE_F16) return LMRS_ERR_DTYPE;
  if (world <= 0 || world > lmrs::kArMaxRanks || rank < 0 || rank >= world || rows < 0 ||
      H <= 0 || H % 8 || H > lmrs::kArnMaxCluster * lmrs::kArnMaxVecs * lmrs::kArnCols ||
      max_elems / 2 > static_cast<size_t>(INT32_MAX) ||
      static_cast<size_t>(rows) * static_cast<size_t>(H) > max_elems)
    return LMRS_ERR_SHAPE;
  if (rows == 0) return LMRS_OK;
  if (!outp || !residual || !partial || !weight || !buffers) return LMRS_ERR_NULL;
  for (int r = 0; r < world; ++r)
    if (!buffers[r]) return LMRS_ERR_NULL;
  if (!aligned16(outp) || !aligned16(residual) || !aligned16(partial) || !aligned16(weight))
    return LMRS_ERR_ALIGN;
  return -1;  // arguments fine: launch
}

}  // namespace

extern "C" {

LMRS_API int lmrs_allreduce_rmsnorm(void* out, void* residual, const void* partial,
                                    const void* weight, int rows, int H, float eps, int dtype,
                                    int rank, int world, void* const* buffers, size_t max_elems,
                                    lmrs_stream_t stream) {
  int rc = allreduce_norm_check(out, residual, partial, weight, rows, H, dtype, rank, world,
                                buffers, max_elems);
  if (rc >= 0) return rc;
  int dev = 0;
  if ((rc = check_device(&dev))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? allreduce_norm_launch<__nv_bfloat16, false>(out, nullptr, nullptr, residual,
                                                           partial, weight, rows, H, eps, rank,
                                                           world, buffers, max_elems, st, dev)
             : allreduce_norm_launch<__half, false>(out, nullptr, nullptr, residual, partial,
                                                    weight, rows, H, eps, rank, world, buffers,
                                                    max_elems, st, dev);
}

LMRS_API int lmrs_allreduce_rmsnorm_fp8(uint8_t* q_out, float* scale_out, void* residual,
                                        const void* partial, const void* weight, int rows, int H,
                                        float eps, int dtype, int rank, int world,
                                        void* const* buffers, size_t max_elems,
                                        lmrs_stream_t stream) {
  int rc = allreduce_norm_check(q_out, residual, partial, weight, rows, H, dtype, rank, world,
                                buffers, max_elems);
  if (rc >= 0) return rc;
  if (!scale_out) return LMRS_ERR_NULL;
  int dev = 0;
  if ((rc = check_device(&dev))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? allreduce_norm_launch<__nv_bfloat16, true>(nullptr, q_out, scale_out, residual,
                                                          partial, weight, rows, H, eps, rank,
                                                          world, buffers, max_elems, st, dev)
             : allreduce_norm_launch<__half, true>(nullptr, q_out, scale_out, residual, partial,
                                                   weight, rows, H, eps, rank, world, buffers,
                                                   max_elems, st, dev);
}


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
