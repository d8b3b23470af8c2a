// lmrs_capi.cu — the C-ABI (include/lmrs_quant.h) and host-side dispatch.
//
// Unity translation unit: every kernel header is included here so the device
// error word (lmrs::g_device_error) is one symbol without relocatable device
// code.  Host responsibilities, mirroring the reference's `kernels::linear`
// (crates/kernels/src/tensor_ops.rs:225-246) plus what the reference leaves
// unchecked (kernels/ffi/tensor_ffi.cu:830-840 ignores a bad dtype silently):
//   * argument validation -> int status, nothing launched on rejection;
//   * dispatch by M: register-dequant tensor-core GEMV (decode) or tcgen05 GEMM
//     (prefill);
//   * TMA tensor maps (cuTensorMapEncodeTiled via the runtime's driver entry
//     point, so the library has no link-time libcuda dependency);
//   * cluster launches (cudaLaunchKernelEx) for the split-K GEMVs.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "lmrs_quant.h"
#include "awq_gemm_swap.cuh"
#include "awq_gemv.cuh"
#include "awq_gemv4.cuh"
#include "awq_i8.cuh"
#include "awq_pack.cuh"
#include "fp8_kernels.cuh"
#include "lmrs_ptx.cuh"
#include "tc_gemm.cuh"
#include "tc_gemm2.cuh"
#include "fp8_swap.cuh"
#include "awq_tmem.cuh"
#include "awq_gemm_tmem.cuh"
#include "awq_gemm_pair.cuh"
#include "fp8_gemm_pair.cuh"

namespace {

constexpr int kVersion = 1;
constexpr int kMaxDevices = 64;
thread_local int t_last_cuda_error = 0;

// ---- tuning knobs (lmrs_set_tuning); defaults chosen from B200 measurements
struct Tuning {
  int awq_gemv_max_m = 16;   // M up to this -> register-dequant GEMV (16 at most)
  int awq_swap_max_m = 64;   // M up to this -> swap-AB split-K tcgen05 while N/128 < SMs; above -> tile GEMM
  int awq_swap_deep_k = 5;   // ... and up to 128 tokens on any N when 4K >= this x N (0 = off)
  int fp8_gemv_max_m = 8;    // M up to this (and K*N up to fp8_gemv_max_kn) -> register-fed FP8 GEMV
  int fp8_gemv_max_kn = 1 << 25;  // larger weights: the swap-AB kernel streams faster
  int fp8_swap_max_m = 64;   // M up to this -> swap-AB tcgen05 FP8 (64 at most)
  int fp8_swap_cluster = 0;  // 0 = heuristic
  int fp8_swap_deep_k = 4;   // decode FP8: swap-AB instead of the GEMV when K >= this x N (0 = off)
  int gemv_ctas_per_sm = 4;  // resident CTAs per SM the GEMV grids are sized for
  int awq_gemv_cluster = 0;  // 0 = heuristic
  int awq_swap_cluster = 0;  // 0 = heuristic
  int awq_swap_narrow_tiles = 32;  // swap-AB up to 128 tokens while N / 128 <= this (0 = off)
  int awq_gemm_pair = 0;     // 1: CTA-pair (cta_group::2) GEMM for large M; 0: one-SM tiles
  int gemm_bn = 256;         // one-SM GEMM tile width: 256 or 224; 0 = pick by wave count
  int fp8_gemv_cluster = 0;
  // all-reduce: the two-stage (reduce-scatter + all-gather) kernel from this many
  // ranks and elements (the one-shot kernel pushes world x n packets per rank).
  // TP=8 decode steps: config 4 at batch 32 (262144 elements) 10.34 -> 8.73 ms,
  // config 3 at batch 64 3.86 -> 3.26 ms; at 65536 elements (config 3, batch 16)
  // the one-shot kernel fused into the norm stays ahead (2.22 vs 2.28 ms)
  int ar_two_stage_min_world = 4;
  int ar_two_stage_min_elems = 131072;
  // FP8 GEMM tile order: groups of this many M tiles walked N tile by N tile.
  // Graph-timed at M = 2048..8192 on the config-2 shapes, 32 beat 8 by 1-4 %
  // (4096 x 28672 at 8192: 838.8 vs 846.6 us; 14336 x 4096: 354.6 vs 364.9).
  int fp8_gemm_group_m = 32;
  // 128-wide FP8 GEMM tiles while that grid still fits one wave (M = 512 on
  // N = 4096: 64 256-wide tiles, 27.7 -> 19.7 us; 14336 x 4096 67.1 -> 52.9);
  // past one wave they lose (M = 1024, 14336 x 4096: 92.9 vs 67.6 us)
  int fp8_gemm_bn128 = 1;
  // CTA-pair (cta_group::2) 256 x 256 FP8 tiles from fp8_gemm_pair_min_m tokens
  // where 128-wide one-SM tiles do not fit one wave: config 2 at M = 8192 852.6 ->
  // 769.9 us (4096 x 28672), 123.6 -> 113.6 (4096 x 4096), 380.0 -> 345.7 (14336 x
  // 4096), 4096 x 28672 at M = 256 49.9 -> 46.6; bit-identical to the one-SM kernel
  int fp8_gemm_pair = 1;
  int fp8_gemm_pair_min_m = 256;
  int fp8_gemm_pair_ksub = 2;   // its K stage: 1 = 128 bytes (6-deep ring), 2 = 256 bytes (3-deep)
  int pdl = 1;               // programmatic dependent launch on every kernel
  int awq_gemv_slots = 4;    // ring slots of the AWQ GEMV (even, 2..8)
  int awq_gemv4 = 1;         // M <= 4: the permute-free GEMV (0: the general one)
  int gemv_box_rows = 128;   // TMA GEMV box height (128 or 64; 64 forced for group 64)
  int awq_gemv4_slots = 4;   // its ring slots (4 or 8)
  int attn_stages = 3;       // decode attention cp.async ring depth (2..4)
  int attn_ctas_per_sm = 2;  // decode attention context split target
  int attn_global_merge = 1; // small batches: several clusters of splits, merged through the workspace
  int attn_multi_min_ctx = 2048;  // ... only above this context (fewer, longer splits win below)
  int awq_tmem_min_m = 9;    // TMEM-staged tcgen05 AWQ linear for M in [min, max];
  int awq_tmem_max_m = 32;   // its cost is flat in M (32 at most)
  int awq_tmem_min_m_wide = 5;  // ... and down to this M when N >= K (0 = off)
  int awq_tmem_cluster = 0;  // 0 = heuristic
  int awq_tmem_ctas_per_sm = 2;
  int awq_gemm_tmem = 1;     // prefill: GEMM with the weights as the TMEM A operand (0: smem-staged)
  int awq_gemm_tmem_bt = 256;  // its token tile (128, 192 or 256; 256 measured fastest at every M)
  int awq_gemm_tmem_bk = 128;  // its K-block depth at 256 tokens (128 where K and the group allow; 64)
  int awq_gemm_tmem_pair = 0;  // above 128 tokens, N % 256 == 0: the CTA-pair (cta_group::2) form
  int awq_i8_max_m = 1;      // M up to this (2 at most): packed bytes as integer MMA operands
  int awq_i8_slots = 5;      // its ring slots at most (fewer when the grid fills the SMs)
  int awq_i8_ctas_per_sm = 2;
  int awq_i8_cluster = 0;    // 0 = heuristic (1..8)
  int awq_i8_box_rows = 128; // its box height for groups of 128k rows (128 or 64)
  int decode_layer_trace = 0;  // 1: lmrs_fp8_decode_layer writes per-phase timestamps (workspace tail)
};
Tuning g_tune;

int record(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return LMRS_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- per-device checks (cached)
std::atomic<int> g_dev_ok[kMaxDevices];  // 0 unknown, 1 ok, -1 not sm_100

int check_device(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record(e);
  if (dev < 0 || dev >= kMaxDevices) return LMRS_ERR_DEVICE;
  int st = g_dev_ok[dev].load(std::memory_order_relaxed);
  if (st == 0) {
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return record(e);
    st = (major == 10) ? 1 : -1;
    g_dev_ok[dev].store(st, std::memory_order_relaxed);
  }
  if (dev_out) *dev_out = dev;
  return st == 1 ? LMRS_OK : LMRS_ERR_DEVICE;
}

// ---- SM count per device (persistent grids)
std::atomic<int> g_sm_count[kMaxDevices];

int sm_count(int dev) {
  int v = g_sm_count[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    g_sm_count[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

int sm_count_cached() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  return sm_count(dev);
}

// ---- dynamic shared memory opt-in, once per (kernel, device)
template <typename K>
int ensure_smem(K kernel, int bytes, std::atomic<int>* done, int dev) {
  if (done[dev].load(std::memory_order_acquire) >= bytes) return LMRS_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return record(e);
  done[dev].store(bytes, std::memory_order_release);
  return LMRS_OK;
}

// The same with the per-device record kept per kernel instantiation (Kern is
// the kernel itself, so every template instance has its own).
template <auto Kern>
int ensure_smem_of(int bytes, int dev) {
  static std::atomic<int> done[kMaxDevices];
  return ensure_smem(Kern, bytes, done, dev);
}

// ---- TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tensor map: dim0 innermost (contiguous), row stride in bytes.
int make_tmap(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0,
              uint64_t dim1, uint64_t row_bytes, uint32_t box0, uint32_t box1,
              CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMRS_ERR_CUDA;
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return LMRS_ERR_CUDA;
  }
  return LMRS_OK;
}

int after_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LMRS_OK : record(e);
}

int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Launch with a cluster dimension (0 = no cluster attribute) and, when the
// `pdl` knob is on, programmatic stream serialisation (the kernel may start
// while its predecessor drains; every kernel here waits with griddepcontrol
// before touching its activations or writing global memory).
template <typename Kern, typename... Args>
int launch_ex(Kern kernel, int grid_x, int cluster, int threads, int smem, cudaStream_t stream,
              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_x, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (g_tune.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return record(e);
  return LMRS_OK;
}

// 2-D/3-D grid, no cluster, programmatic dependent launch when enabled.
template <typename Kern, typename... Args>
int launch_ex_grid(Kern kernel, dim3 grid, int threads, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (g_tune.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    n = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return record(e);
  return LMRS_OK;
}

// 2-D/3-D grid with a thread-block cluster shape, PDL when enabled.
template <typename Kern, typename... Args>
int launch_ex_cluster3(Kern kernel, dim3 grid, dim3 cluster, int threads, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = cluster.x;
  attr[n].val.clusterDim.y = cluster.y;
  attr[n].val.clusterDim.z = cluster.z;
  ++n;
  if (g_tune.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return record(e);
  return LMRS_OK;
}

template <typename Kern, typename... Args>
int launch_cluster(Kern kernel, int grid_x, int cluster, int threads, int smem,
                   cudaStream_t stream, Args... args) {
  return launch_ex(kernel, grid_x, cluster, threads, smem, stream, args...);
}

std::atomic<int> g_smem_f8_gemm[kMaxDevices];
std::atomic<int> g_smem_f8_gemv[3][kMaxDevices];

// ------------------------------------------------------------------ AWQ
// Every AWQ launcher is a template on the activation type T (__half for
// LMRS_DTYPE_F16, __nv_bfloat16 for LMRS_DTYPE_BF16): x, y and bias are T, the
// scales stay fp16, and the kernels dequantise to T (lmrs_ptx.cuh, Act<T>).

// Cluster size for a TMA-fed GEMV: split K over C CTAs so that every CTA of
// the grid is resident at once (~4 per SM), C <= 8 and C <= K units.
int gemv_cluster(int strips, int units, int forced) {
  int C = forced > 0 ? forced : (sm_count_cached() * g_tune.gemv_ctas_per_sm) / (strips > 0 ? strips : 1);
  C = clampi(C, 1, 8);
  if (C > units) C = units > 0 ? units : 1;
  return C;
}

// Power-of-two cluster size for the AWQ GEMV (its reduction splits the strip's
// 128 columns evenly over the cluster).
int pow2_floor(int v) {
  int r = 1;
  while (r * 2 <= v) r *= 2;
  return r;
}

template <int MT, int BR, typename T>
int awq_gemv_launch_t(const CUtensorMap& tq, const CUtensorMap& tx, const CUtensorMap& ts,
                      const CUtensorMap& tz, T* y, const T* bias, int M, int K, int N, int group,
                      cudaStream_t stream, int dev, int strips, int C, int S) {
  using L = lmrs::AwqGemvLayout<MT, BR>;
  const int smem = L::smem_bytes(S);
  int rc;
  if ((rc = ensure_smem_of<lmrs::awq_gemv_kernel<MT, BR, T>>(smem, dev))) return rc;
  rc = launch_ex(lmrs::awq_gemv_kernel<MT, BR, T>, strips * C, C, lmrs::kAwqGemvThreads, smem,
                 stream, tq, tx, ts, tz, y, bias, M, K, N, group, S);
  return rc ? rc : after_launch();
}

template <int BR, typename T>
int awq_gemv4_launch_t(const CUtensorMap& tq, const CUtensorMap& tx, const CUtensorMap& ts,
                       const CUtensorMap& tz, T* y, const T* bias, int M, int K, int N, int group,
                       cudaStream_t stream, int dev, int strips, int C, int S) {
  const int smem = lmrs::AwqGemv4Layout<BR>::smem_bytes(S);
  int rc;
  if ((rc = ensure_smem_of<lmrs::awq_gemv4_kernel<BR, T>>(smem, dev))) return rc;
  rc = launch_ex(lmrs::awq_gemv4_kernel<BR, T>, strips * C, C, lmrs::kAwqGemv4Threads, smem,
                 stream, tq, tx, ts, tz, y, bias, M, K, N, group, S);
  return rc ? rc : after_launch();
}

template <int NT, typename T>
int awq_tmem_launch_t(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                      const T* bias, int M, int K, int N, int group, cudaStream_t stream,
                      int dev) {
  using L = lmrs::AtLayout<NT>;
  const int strips = (N + lmrs::kAtCols - 1) / lmrs::kAtCols;
  const int nb_all = K / lmrs::kAtRows;
  int C = g_tune.awq_tmem_cluster > 0
              ? g_tune.awq_tmem_cluster
              : (g_tune.awq_tmem_ctas_per_sm * sm_count(dev)) / (strips > 0 ? strips : 1);
  C = pow2_floor(clampi(C, 1, lmrs::kAtMaxCluster));
  while (C > 1 && C > nb_all) C /= 2;
  CUtensorMap tq, tx, ts, tz;
  int rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      lmrs::kAtWords, lmrs::kAtRows, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, 64, NT,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, N, K / group, uint64_t(N) * 2,
                      lmrs::kAtCols, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, N / 8, K / group,
                      uint64_t(N / 8) * 4, lmrs::kAtWords, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  constexpr int smem = L::kSmem;
  if ((rc = ensure_smem_of<lmrs::awq_tmem_kernel<NT, T>>(smem, dev))) return rc;
  rc = launch_ex(lmrs::awq_tmem_kernel<NT, T>, strips * C, C, lmrs::kAtThreads, smem, stream, tq,
                 tx, ts, tz, y, bias, M, K, N, group);
  return rc ? rc : after_launch();
}

// 9..16 tokens: the register-fed GEMV is faster unless N is wide; 17..32: the
// TMEM-staged kernel (flat in M) beats both the GEMV and the swap-AB kernel.
// Measured graph-timed on the 8B/config-1 shapes: from 9 tokens the TMEM kernel
// beats the register-fed GEMV on every shape (4096 x 4096 at 16: 7.7 vs 9.2 us);
// at 5..8 it wins where N >= K and loses on deep-K, narrow-N shapes (14336 x
// 4096: 20.5 vs 19.5 us); at 3..4 the four-token GEMV is ahead everywhere.
bool awq_use_tmem(int M, int K, int N) {
  if (M > g_tune.awq_tmem_max_m || M > 32) return false;
  if (M >= g_tune.awq_tmem_min_m) return true;
  return g_tune.awq_tmem_min_m_wide > 0 && M >= g_tune.awq_tmem_min_m_wide && N >= K;
}

// 33..128 tokens, measured graph-timed: the split-K swap-AB kernel wins while the
// prefill GEMM has few 128-channel tiles and a deep K to walk per tile (14336 x
// 4096 at 96 tokens: 60 vs 92 us; 28672 x 8192: 122 vs 180), the GEMM once the
// tiles fill the SMs (4096 x 28672 at 40..64 tokens: 44 vs 51-54 us; 8192 x
// 57344: 156 vs 172) or the tokens pass 64 on shallow K (4096 x 14336 at 96: 33
// vs 54 us).  The crossover in K / N at 96-128 tokens lies between 1 (4096 x
// 4096: GEMM 30.7 vs 31.4 us) and 1.33 (4096 x 3072: swap 21.6 vs 30.6 us), so
// swap from K >= 1.25 N.  With the split-K clusters sized to a power of two,
// narrow outputs (at most awq_swap_narrow_tiles 128-channel tiles) take swap-AB
// up to 128 tokens as well (bf16, 4096 x 4096 at 96 / 128 tokens: 17.1 / 18.5 us
// against 27.3 / 27.6 for the tile GEMM; 4096 x 6144, 48 tiles, stays on the GEMM:
// 27.8 against 29.8).
bool awq_use_swap(int M, int K, int N, int sms) {
  if (M > 128) return false;
  if (g_tune.awq_swap_deep_k > 0 &&
      4LL * K >= static_cast<long long>(g_tune.awq_swap_deep_k) * N)
    return true;
  const int tiles = (N + lmrs::kAgtCh - 1) / lmrs::kAgtCh;
  if (tiles <= g_tune.awq_swap_narrow_tiles) return true;
  return M <= g_tune.awq_swap_max_m && tiles < sms;
}

template <typename T>
int awq_tmem_launch(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                    const T* bias, int M, int K, int N, int group, cudaStream_t stream, int dev) {
  if (M <= 16) return awq_tmem_launch_t<16, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  return awq_tmem_launch_t<32, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
}

template <int TOK, int BR, typename T>
int awq_i8_launch_t(const CUtensorMap& tq, const CUtensorMap& ts, const CUtensorMap& tz,
                    const T* x, T* y, const T* bias, int M, int K, int N, int group,
                    cudaStream_t stream, int dev, int strips, int C, int S, int nbmax) {
  using L = lmrs::AwqI8Layout<TOK, BR>;
  // Slots: as many as asked (up to the CTA's box count) while the grid takes at
  // most 80 % of the CTAs that fit per SM at that size, so that the next kernel
  // can become resident early (programmatic dependent launch); at least 2.
  const int ctas = strips * C;
  auto fits = [&](int s) {
    const int smem = L::smem_bytes(s);
    const int per_sm = smem <= 227 * 1024 ? (228 * 1024) / (smem + 1024) : 0;
    return per_sm > 0 && ctas * 5 <= per_sm * sm_count(dev) * 4;
  };
  if (S > nbmax) S = nbmax;
  while (S > 2 && !fits(S)) --S;
  while (S > 2 && L::smem_bytes(S) > 227 * 1024) --S;
  const int smem = L::smem_bytes(S);
  if (smem > 227 * 1024) return -1;
  CUtensorMap tx;
  int rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, BR, TOK,
                      CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = ensure_smem_of<lmrs::awq_gemv_i8_kernel<TOK, BR, T>>(smem, dev))) return rc;
  rc = launch_ex(lmrs::awq_gemv_i8_kernel<TOK, BR, T>, ctas, C, lmrs::kI8Threads, smem, stream, tq,
                 ts, tz, tx, y, bias, M, K, N, group, S);
  return rc ? rc : after_launch();
}

// 1-2 tokens with the packed bytes as integer MMA operands.  Returns -1 when
// the shape does not fit the kernel (the caller then takes the 16-bit GEMV).
template <typename T>
int awq_i8_launch(T* y, const T* x, const int32_t* qw, const uint32_t* qz, const __half* sc,
                  const T* bias, int M, int K, int N, int group, cudaStream_t stream, int dev) {
  const int BR = group % 128 == 0 && g_tune.awq_i8_box_rows != 64 ? 128 : 64;
  if (M < 1 || M > 2 || K % BR) return -1;
  const int strips = (N + lmrs::kI8Strip - 1) / lmrs::kI8Strip;
  const int nb_all = K / BR;
  int C = g_tune.awq_i8_cluster > 0
              ? g_tune.awq_i8_cluster
              : (sm_count(dev) * clampi(g_tune.awq_i8_ctas_per_sm, 1, 4)) / strips;
  C = clampi(C, 1, lmrs::kI8MaxCluster);
  if (C > nb_all) C = nb_all;
  const int nbmax = (nb_all + C - 1) / C;
  const int S = clampi(g_tune.awq_i8_slots, 2, 12);
  CUtensorMap tq, ts, tz;
  int rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      lmrs::kI8Words, BR, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, N, K / group, uint64_t(N) * 2,
                      lmrs::kI8Strip, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, N / 8, K / group,
                      uint64_t(N / 8) * 4, lmrs::kI8Words, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if (M == 1 && BR == 128)
    return awq_i8_launch_t<1, 128, T>(tq, ts, tz, x, y, bias, M, K, N, group, stream, dev, strips,
                                      C, S, nbmax);
  if (M == 1)
    return awq_i8_launch_t<1, 64, T>(tq, ts, tz, x, y, bias, M, K, N, group, stream, dev, strips,
                                     C, S, nbmax);
  if (BR == 128)
    return awq_i8_launch_t<2, 128, T>(tq, ts, tz, x, y, bias, M, K, N, group, stream, dev, strips,
                                      C, S, nbmax);
  return awq_i8_launch_t<2, 64, T>(tq, ts, tz, x, y, bias, M, K, N, group, stream, dev, strips, C,
                                   S, nbmax);
}

template <typename T>
int awq_gemv_launch(T* y, const T* x, const int32_t* qw, const uint32_t* qz, const __half* sc,
                    const T* bias, int M, int K, int N, int group, cudaStream_t stream, int dev) {
  if (M <= g_tune.awq_i8_max_m) {
    const int rc = awq_i8_launch<T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
    if (rc >= 0) return rc;
  }
  const int BR = (group % 128 == 0 && g_tune.gemv_box_rows != 64) ? 128 : 64;
  const int MT = M <= 8 ? 1 : 2;
  const int strips = (N + lmrs::kAwqGemvStrip - 1) / lmrs::kAwqGemvStrip;
  const int nb_all = K / BR;
  int C;
  if (g_tune.awq_gemv_cluster > 0) {
    C = pow2_floor(clampi(g_tune.awq_gemv_cluster, 1, lmrs::kAwqGemvMaxCluster));
  } else {
    const int cps = MT == 1 ? g_tune.gemv_ctas_per_sm : 3;
    C = pow2_floor(clampi((sm_count(dev) * cps) / strips, 1, lmrs::kAwqGemvMaxCluster));
  }
  while (C > 1 && C > nb_all) C /= 2;
  const int per_cta = (nb_all + C - 1) / C;
  int S = clampi(g_tune.awq_gemv_slots, 2, 8) & ~1;   // even: two box streams per CTA
  if (S > ((per_cta + 1) & ~1)) S = (per_cta + 1) & ~1;
  if (S < 2) S = 2;
  CUtensorMap tq, tx, ts, tz;
  int rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      lmrs::kAwqGemvWords, BR, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, 64, 8 * MT,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, N, K / group, uint64_t(N) * 2,
                      lmrs::kAwqGemvStrip, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, N / 8, K / group,
                      uint64_t(N / 8) * 4, lmrs::kAwqGemvWords, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if (M <= 4 && g_tune.awq_gemv4) {
    int S4 = g_tune.awq_gemv4_slots >= 16 ? 16 : (g_tune.awq_gemv4_slots >= 8 ? 8 : 4);
    while (S4 > 4 && per_cta <= S4 / 2) S4 /= 2;
    if (BR == 128)
      return awq_gemv4_launch_t<128, T>(tq, tx, ts, tz, y, bias, M, K, N, group, stream, dev,
                                        strips, C, S4);
    return awq_gemv4_launch_t<64, T>(tq, tx, ts, tz, y, bias, M, K, N, group, stream, dev, strips,
                                     C, S4);
  }
  if (MT == 1 && BR == 128)
    return awq_gemv_launch_t<1, 128, T>(tq, tx, ts, tz, y, bias, M, K, N, group, stream, dev,
                                        strips, C, S);
  if (MT == 2 && BR == 128)
    return awq_gemv_launch_t<2, 128, T>(tq, tx, ts, tz, y, bias, M, K, N, group, stream, dev,
                                        strips, C, S);
  if (MT == 1)
    return awq_gemv_launch_t<1, 64, T>(tq, tx, ts, tz, y, bias, M, K, N, group, stream, dev,
                                       strips, C, S);
  return awq_gemv_launch_t<2, 64, T>(tq, tx, ts, tz, y, bias, M, K, N, group, stream, dev, strips,
                                     C, S);
}

template <int NT, typename T>
int awq_swap_launch_nt(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                       const T* bias, int M, int K, int N, int group, cudaStream_t stream,
                       int dev) {
  CUtensorMap tx, tq, ts, tz;
  int rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, lmrs::kSwBK, NT,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      lmrs::kSwBN / 8, lmrs::kSwBK, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, N, K / group, uint64_t(N) * 2,
                      lmrs::kSwBN, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, N / 8, K / group,
                      uint64_t(N / 8) * 4, lmrs::kSwBN / 8, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  constexpr int smem = lmrs::sw_smem_bytes(NT);
  if ((rc = ensure_smem_of<lmrs::awq_gemm_swap_kernel<NT, T>>(smem, dev))) return rc;
  const int tiles = (N + lmrs::kSwBN - 1) / lmrs::kSwBN;
  const int KB = K / lmrs::kSwBK;
  // CTAs resident per SM at this tile width (launch bounds allow 2; the
  // 128-token tile's ~117 KB of shared memory leaves room for one)
  constexpr int per_sm = (228 * 1024) / (smem + 1024) < 2 ? 1 : 2;
  // split-K clusters of a power of two: 4096 x 6144 at 48 tokens took 27.2 us on
  // the 3-CTA clusters the plain quotient gave, 20.9 on 4 and 25.1 on 2
  int C = g_tune.awq_swap_cluster > 0 ? g_tune.awq_swap_cluster
                                      : pow2_floor(clampi((per_sm * sm_count(dev)) / tiles, 1, 8));
  C = clampi(C, 1, 8);
  if (C > KB) C = KB;
  rc = launch_cluster(lmrs::awq_gemm_swap_kernel<NT, T>, tiles * C, C, lmrs::kSwThreads, smem,
                      stream, tx, tq, ts, tz, y, bias, M, K, N, group);
  return rc ? rc : after_launch();
}

template <typename T>
int awq_swap_launch(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                    const T* bias, int M, int K, int N, int group, cudaStream_t stream, int dev) {
  if (M <= 16) return awq_swap_launch_nt<16, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  if (M <= 32) return awq_swap_launch_nt<32, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  if (M <= 64) return awq_swap_launch_nt<64, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  return awq_swap_launch_nt<128, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
}

template <int BT, int BK, typename T>
int awq_gemm_tmem_launch_t(T* y, const T* x, const int32_t* qw, const int32_t* qz,
                           const __half* sc, const T* bias, int M, int K, int N, int group,
                           cudaStream_t stream, int dev) {
  using L = lmrs::AgtLayout<BT, BK>;
  CUtensorMap tx, tq;
  int rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, 64, BT,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      lmrs::kAgtWords, BK, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  if ((rc = ensure_smem_of<lmrs::awq_gemm_tmem_kernel<BT, BK, T>>(L::kSmem, dev))) return rc;
  const int tiles = ((N + lmrs::kAgtCh - 1) / lmrs::kAgtCh) * ((M + BT - 1) / BT);
  const int grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
  rc = launch_ex(lmrs::awq_gemm_tmem_kernel<BT, BK, T>, grid, 0, L::kThreads, L::kSmem,
                 stream, tx, tq, sc, reinterpret_cast<const uint32_t*>(qz), y, bias, M, K, N,
                 group);
  return rc ? rc : after_launch();
}

template <typename T>
int awq_gemm_tmem_launch(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                         const T* bias, int M, int K, int N, int group, cudaStream_t stream,
                         int dev) {
  const int f = g_tune.awq_gemm_tmem_bt;
  const int bt = (f == 128 || f == 192) ? f : 256;
  if (bt == 128)
    return awq_gemm_tmem_launch_t<128, 64, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  if (bt == 192)
    return awq_gemm_tmem_launch_t<192, 64, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  // 128-deep K-blocks where every K-block lies in one quantisation group
  if (g_tune.awq_gemm_tmem_bk != 64 && K % 128 == 0 && group % 128 == 0)
    return awq_gemm_tmem_launch_t<256, 128, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  return awq_gemm_tmem_launch_t<256, 64, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
}

// CTA-pair version of the prefill GEMM (256 channels x 256 tokens per pair).
template <typename T>
int awq_gemm_pair_launch(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                         const T* bias, int M, int K, int N, int group, cudaStream_t stream,
                         int dev) {
  using L = lmrs::ApLayout;
  CUtensorMap tx, tq;
  int rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      lmrs::kAgtWords, lmrs::kAgtBK, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  if ((rc = ensure_smem_of<lmrs::awq_gemm_pair_kernel<T>>(L::kSmem, dev))) return rc;
  const int tiles = ((N + lmrs::kApCh - 1) / lmrs::kApCh) * ((M + lmrs::kApBT - 1) / lmrs::kApBT);
  const int max_pairs = sm_count(dev) / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  rc = launch_cluster(lmrs::awq_gemm_pair_kernel<T>, 2 * pairs, 2, lmrs::kApThreads, L::kSmem,
                      stream, tx, tq, sc, reinterpret_cast<const uint32_t*>(qz), y, bias, M, K, N,
                      group);
  return rc ? rc : after_launch();
}

template <typename T>
int awq_gemm2_launch(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                     const T* bias, int M, int K, int N, int group, cudaStream_t stream, int dev) {
  CUtensorMap tx, tq, ts, tz;
  int rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4, 16,
                      64, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, N, K / group, uint64_t(N) * 2,
                      128, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, N / 8, K / group,
                      uint64_t(N / 8) * 4, 16, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = ensure_smem_of<lmrs::awq_gemm_tc2_kernel<T>>(lmrs::kP2SmemBytes, dev))) return rc;
  const int tiles = ((N + lmrs::kP2BN - 1) / lmrs::kP2BN) * ((M + lmrs::kP2BM - 1) / lmrs::kP2BM);
  const int pairs = tiles < sm_count(dev) / 2 ? tiles : sm_count(dev) / 2;
  rc = launch_cluster(lmrs::awq_gemm_tc2_kernel<T>, 2 * pairs, 2, lmrs::kP2Threads,
                      lmrs::kP2SmemBytes, stream, tx, tq, ts, tz, y, bias, M, K, N, group);
  return rc ? rc : after_launch();
}

// Tile width for the one-SM tcgen05 GEMMs: 256 by default (measured fastest on
// B200 for the config shapes); 224 can be forced, and 0 picks the width with the
// fewer tile-columns x waves (a 224-wide tile costs more than 224/256 of a
// 256-wide one, so the wave count alone mispredicts).
int pick_bn(int M, int N, int sms) {
  if (g_tune.gemm_bn == 256 || g_tune.gemm_bn == 224) return g_tune.gemm_bn;
  long best_cost = -1;
  int best = 256;
  for (int bn : {256, 224}) {
    const long tiles = long((N + bn - 1) / bn) * ((M + lmrs::kTcBM - 1) / lmrs::kTcBM);
    const long waves = (tiles + sms - 1) / sms;
    const long cost = waves * bn;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <int BN, typename T>
int awq_gemm_launch_bn(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                       const T* bias, int M, int K, int N, int group, cudaStream_t stream,
                       int dev) {
  CUtensorMap tx, tq, ts, tz;
  int rc;
  if ((rc = make_tmap(&tx, lmrs::Act<T>::kTma, x, K, M, uint64_t(K) * 2, 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, N / 8, K, uint64_t(N / 8) * 4,
                      BN / 8, 64, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, N, K / group, uint64_t(N) * 2,
                      BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, N / 8, K / group,
                      uint64_t(N / 8) * 4, BN / 8, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  constexpr int smem = lmrs::AwqTile<BN>::kSmem;
  if ((rc = ensure_smem_of<lmrs::awq_gemm_tc_kernel<BN, T>>(smem, dev))) return rc;
  const int tiles = ((N + BN - 1) / BN) * ((M + lmrs::kTcBM - 1) / lmrs::kTcBM);
  const int grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
  rc = launch_ex(lmrs::awq_gemm_tc_kernel<BN, T>, grid, 0, lmrs::kAwqGemmThreads, smem, stream,
                 tx, tq, ts, tz, y, bias, M, K, N, group);
  return rc ? rc : after_launch();
}

template <typename T>
int awq_gemm_launch(T* y, const T* x, const int32_t* qw, const int32_t* qz, const __half* sc,
                    const T* bias, int M, int K, int N, int group, cudaStream_t stream, int dev) {
  if (pick_bn(M, N, sm_count(dev)) == 224)
    return awq_gemm_launch_bn<224, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
  return awq_gemm_launch_bn<256, T>(y, x, qw, qz, sc, bias, M, K, N, group, stream, dev);
}

// Dispatch by M (every regime for both activation types).
template <typename T>
int awq_linear_dispatch(T* y, const T* x, const int32_t* qweight, const int32_t* qzeros,
                        const __half* sc, const T* bias, int M, int K, int N, int group,
                        cudaStream_t st, int dev) {
  if (awq_use_tmem(M, K, N))
    return awq_tmem_launch<T>(y, x, qweight, qzeros, sc, bias, M, K, N, group, st, dev);
  if (M <= g_tune.awq_gemv_max_m && M <= 16)
    return awq_gemv_launch<T>(y, x, qweight, reinterpret_cast<const uint32_t*>(qzeros), sc, bias,
                              M, K, N, group, st, dev);
  if (awq_use_swap(M, K, N, sm_count(dev)))
    return awq_swap_launch<T>(y, x, qweight, qzeros, sc, bias, M, K, N, group, st, dev);
  // up to one token tile, more 128-channel tiles than SMs leave a tail wave the
  // 256-channel smem-staged tiles avoid
  if (g_tune.awq_gemm_tmem && (M > 128 || (N + lmrs::kAgtCh - 1) / lmrs::kAgtCh <= sm_count(dev))) {
    if (g_tune.awq_gemm_tmem_pair && M > 128 && N % lmrs::kApCh == 0)
      return awq_gemm_pair_launch<T>(y, x, qweight, qzeros, sc, bias, M, K, N, group, st, dev);
    return awq_gemm_tmem_launch<T>(y, x, qweight, qzeros, sc, bias, M, K, N, group, st, dev);
  }
  if (g_tune.awq_gemm_pair)
    return awq_gemm2_launch<T>(y, x, qweight, qzeros, sc, bias, M, K, N, group, st, dev);
  return awq_gemm_launch<T>(y, x, qweight, qzeros, sc, bias, M, K, N, group, st, dev);
}

// ------------------------------------------------------------------ FP8
int fp8_quant_launch(uint8_t* q, float* s, const void* x, int rows, int K, int dt,
                     cudaStream_t stream) {
  if (rows == 0) return LMRS_OK;
  int rc = LMRS_OK;
  switch (dt) {
    case LMRS_DTYPE_BF16:
      rc = launch_ex(lmrs::fp8_quant_rows_kernel<0>, rows, 0, lmrs::kQuantThreads, 0, stream, q, s,
                     static_cast<const __nv_bfloat16*>(x), K);
      break;
    case LMRS_DTYPE_F16:
      rc = launch_ex(lmrs::fp8_quant_rows_kernel<1>, rows, 0, lmrs::kQuantThreads, 0, stream, q, s,
                     static_cast<const __half*>(x), K);
      break;
    default:
      rc = launch_ex(lmrs::fp8_quant_rows_kernel<2>, rows, 0, lmrs::kQuantThreads, 0, stream, q, s,
                     static_cast<const float*>(x), K);
      break;
  }
  return rc ? rc : after_launch();
}

int fp8_gemv_launch(__nv_bfloat16* y, const uint8_t* xq, const float* sx, const uint8_t* wq,
                    const float* sw, const __nv_bfloat16* bias, int M, int K, int N,
                    cudaStream_t stream, int dev) {
  const int strips = (N + lmrs::kF8GemvRows - 1) / lmrs::kF8GemvRows;
  const int units = (K + 127) / 128;
  // power-of-two cluster: the owner slices of the 64 channels are equal
  int C = pow2_floor(gemv_cluster(strips, units, g_tune.fp8_gemv_cluster));
  while (C > 1 && C > units) C /= 2;
  const int per_cta = (units + C - 1) / C;
  const int MT = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  const int max_ring = lmrs::kF8GemvMaxRing;
  int ring = per_cta < max_ring ? per_cta : max_ring;
  if (ring < 1) ring = 1;
  const int smem = lmrs::f8_gemv_smem_bytes(ring, MT);
  CUtensorMap tw, tx;
  int rc;
  if ((rc = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, K, N, uint64_t(K), 128,
                      lmrs::kF8GemvRows, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, K, M, uint64_t(K), 128, 8 * MT,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (MT == 1) {
    if ((rc = ensure_smem(lmrs::fp8_gemv_kernel<1>, smem, g_smem_f8_gemv[0], dev))) return rc;
    rc = launch_cluster(lmrs::fp8_gemv_kernel<1>, strips * C, C, lmrs::kF8GemvThreads, smem,
                        stream, tw, tx, y, sx, sw, bias, M, K, N, ring);
  } else if (MT == 2) {
    if ((rc = ensure_smem(lmrs::fp8_gemv_kernel<2>, smem, g_smem_f8_gemv[1], dev))) return rc;
    rc = launch_cluster(lmrs::fp8_gemv_kernel<2>, strips * C, C, lmrs::kF8GemvThreads, smem,
                        stream, tw, tx, y, sx, sw, bias, M, K, N, ring);
  } else {
    if ((rc = ensure_smem(lmrs::fp8_gemv_kernel<4>, smem, g_smem_f8_gemv[2], dev))) return rc;
    rc = launch_cluster(lmrs::fp8_gemv_kernel<4>, strips * C, C, lmrs::kF8GemvThreads, smem,
                        stream, tw, tx, y, sx, sw, bias, M, K, N, ring);
  }
  return rc ? rc : after_launch();
}

std::atomic<int> g_smem_f8_gemm224[kMaxDevices];
std::atomic<int> g_smem_f8_gemm128[kMaxDevices];
std::atomic<int> g_smem_f8_pair[2][kMaxDevices];
std::atomic<int> g_smem_f8_swap[3][kMaxDevices];

template <int NT, int ST>
int fp8_swap_launch_t(__nv_bfloat16* y, const uint8_t* xq, const float* sx, const uint8_t* wq,
                      const float* sw, const __nv_bfloat16* bias, int M, int K, int N,
                      cudaStream_t stream, int dev, std::atomic<int>* done) {
  const int strips = (N + lmrs::kFsRows - 1) / lmrs::kFsRows;
  const int units = (K + lmrs::kFsBK - 1) / lmrs::kFsBK;
  int C = g_tune.fp8_swap_cluster > 0 ? g_tune.fp8_swap_cluster
                                      : (2 * sm_count(dev)) / (strips > 0 ? strips : 1);
  C = pow2_floor(clampi(C, 1, lmrs::kFsMaxCluster));
  while (C > 1 && C > units) C /= 2;
  CUtensorMap tw, tx;
  int rc;
  if ((rc = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, K, N, uint64_t(K), lmrs::kFsBK,
                      lmrs::kFsRows, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, K, M, uint64_t(K), lmrs::kFsBK, NT,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  constexpr int smem = lmrs::FsLayout<NT, ST>::kSmem;
  if ((rc = ensure_smem(lmrs::fp8_swap_kernel<NT, ST>, smem, done, dev))) return rc;
  rc = launch_ex(lmrs::fp8_swap_kernel<NT, ST>, strips * C, C, lmrs::kFsThreads, smem, stream, tw,
                 tx, y, sx, sw, bias, M, K, N);
  return rc ? rc : after_launch();
}

int fp8_swap_launch(__nv_bfloat16* y, const uint8_t* xq, const float* sx, const uint8_t* wq,
                    const float* sw, const __nv_bfloat16* bias, int M, int K, int N,
                    cudaStream_t stream, int dev) {
  if (M <= 16)
    return fp8_swap_launch_t<16, 5>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev,
                                    g_smem_f8_swap[0]);
  if (M <= 32)
    return fp8_swap_launch_t<32, 4>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev,
                                    g_smem_f8_swap[1]);
  return fp8_swap_launch_t<64, 3>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev,
                                  g_smem_f8_swap[2]);
}

template <int BN, int KSUB = 1>
int fp8_gemm_launch_bn(__nv_bfloat16* y, const uint8_t* xq, const float* sx, const uint8_t* wq,
                       const float* sw, const __nv_bfloat16* bias, int M, int K, int N,
                       cudaStream_t stream, int dev, std::atomic<int>* smem_done) {
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, K, M, uint64_t(K), 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, K, N, uint64_t(K), 128, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  constexpr int smem = lmrs::F8Tile<BN, KSUB>::kSmem;
  if ((rc = ensure_smem(lmrs::fp8_gemm_tc_kernel<BN, KSUB>, smem, smem_done, dev))) return rc;
  const int tiles = ((N + BN - 1) / BN) * ((M + lmrs::kTcBM - 1) / lmrs::kTcBM);
  const int grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
  const int group_m = g_tune.fp8_gemm_group_m > 0 ? g_tune.fp8_gemm_group_m : 1;
  rc = launch_ex(lmrs::fp8_gemm_tc_kernel<BN, KSUB>, grid, 0, lmrs::kF8Threads, smem, stream, ta, tb, y,
                 sx, sw, bias, M, K, N, group_m);
  return rc ? rc : after_launch();
}

// CTA pairs on 256 x 256 tiles (cluster of 2, no multicast): each CTA's A rows
// and half of B, boxes of 128 rows x 128 bytes.
template <int KSUB>
int fp8_gemm_pair_launch(__nv_bfloat16* y, const uint8_t* xq, const float* sx, const uint8_t* wq,
                         const float* sw, const __nv_bfloat16* bias, int M, int K, int N,
                         cudaStream_t stream, int dev) {
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, K, M, uint64_t(K), 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, K, N, uint64_t(K), 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  constexpr int smem = lmrs::F8Pair<KSUB>::kSmem;
  if ((rc = ensure_smem(lmrs::fp8_gemm_pair_kernel<KSUB>, smem, g_smem_f8_pair[KSUB - 1], dev)))
    return rc;
  const int tiles = ((N + lmrs::kF8PBN - 1) / lmrs::kF8PBN) * ((M + lmrs::kF8PBM - 1) / lmrs::kF8PBM);
  const int pairs = tiles < sm_count(dev) / 2 ? tiles : sm_count(dev) / 2;
  // the one-SM kernel's groups of 128-row tiles, in 256-row bands
  const int group_m = g_tune.fp8_gemm_group_m > 1 ? g_tune.fp8_gemm_group_m / 2 : 1;
  rc = launch_ex(lmrs::fp8_gemm_pair_kernel<KSUB>, 2 * pairs, 2, lmrs::kF8Threads, smem, stream,
                 ta, tb, y, sx, sw, bias, M, K, N, group_m);
  return rc ? rc : after_launch();
}

int fp8_gemm_launch(__nv_bfloat16* y, const uint8_t* xq, const float* sx, const uint8_t* wq,
                    const float* sw, const __nv_bfloat16* bias, int M, int K, int N,
                    cudaStream_t stream, int dev) {
  const int m_tiles = (M + lmrs::kTcBM - 1) / lmrs::kTcBM;
  if (g_tune.fp8_gemm_bn128 && m_tiles * ((N + 127) / 128) <= sm_count(dev))
    return fp8_gemm_launch_bn<128, 2>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev,
                                      g_smem_f8_gemm128);
  if (g_tune.fp8_gemm_pair && M >= g_tune.fp8_gemm_pair_min_m && sm_count(dev) >= 2)
    return g_tune.fp8_gemm_pair_ksub == 2
               ? fp8_gemm_pair_launch<2>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev)
               : fp8_gemm_pair_launch<1>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev);
  if (pick_bn(M, N, sm_count(dev)) == 224)
    return fp8_gemm_launch_bn<224>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev, g_smem_f8_gemm224);
  return fp8_gemm_launch_bn<256>(y, xq, sx, wq, sw, bias, M, K, N, stream, dev, g_smem_f8_gemm);
}

// The tile GEMM's epilogue stores 8 channels at a time (N % 8 == 0); the GEMV
// and swap-AB kernels store single channels.
// Deep, narrow weights (K >= fp8_swap_deep_k x N) stream faster through the
// swap-AB kernel's split-K clusters even when small: a TP=8 rank's merged q/k/v
// of config 4 (8192 x 1280, M = 1) 5.7 us against 6.2 us on the GEMV.
bool fp8_uses_gemv(int M, int K, int N) {
  if (g_tune.fp8_swap_deep_k > 0 &&
      static_cast<int64_t>(K) >= static_cast<int64_t>(g_tune.fp8_swap_deep_k) * N)
    return false;
  return M <= g_tune.fp8_gemv_max_m && M <= 32 &&
         static_cast<int64_t>(K) * N <= static_cast<int64_t>(g_tune.fp8_gemv_max_kn);
}
bool fp8_uses_gemm(int M, int K, int N) {
  return !fp8_uses_gemv(M, K, N) && !(M <= g_tune.fp8_swap_max_m && M <= 64);
}

int fp8_linear_prequant_impl(void* y, const uint8_t* xq, const float* x_scale, const uint8_t* wq,
                             const float* w_scale, const void* bias, int M, int K, int N,
                             cudaStream_t stream, int dev) {
  auto* yb = static_cast<__nv_bfloat16*>(y);
  auto* bb = static_cast<const __nv_bfloat16*>(bias);
  if (fp8_uses_gemv(M, K, N))
    return fp8_gemv_launch(yb, xq, x_scale, wq, w_scale, bb, M, K, N, stream, dev);
  if (M <= g_tune.fp8_swap_max_m && M <= 64)
    return fp8_swap_launch(yb, xq, x_scale, wq, w_scale, bb, M, K, N, stream, dev);
  return fp8_gemm_launch(yb, xq, x_scale, wq, w_scale, bb, M, K, N, stream, dev);
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

// =================================================================== C-ABI
extern "C" {

int lmrs_version(void) { return kVersion; }

const char* lmrs_status_string(int status) {
  switch (status) {
    case LMRS_OK: return "ok";
    case LMRS_ERR_SHAPE: return "invalid shape";
    case LMRS_ERR_DTYPE: return "unsupported dtype";
    case LMRS_ERR_ALIGN: return "pointer not 16-byte aligned";
    case LMRS_ERR_GROUP: return "group size must divide K and be a multiple of 64";
    case LMRS_ERR_WORKSPACE: return "workspace missing or too small";
    case LMRS_ERR_CUDA: return "CUDA call failed";
    case LMRS_ERR_DEVICE: return "current device is not sm_100 (B200)";
    case LMRS_ERR_NULL: return "required pointer is NULL";
    case LMRS_ERR_TIMEOUT: return "kernel wait timed out";
    case LMRS_ERR_TOO_LARGE: return "problem exceeds the no-allocation scratch limit";
    default: return "unknown status";
  }
}

int lmrs_last_cuda_error(void) { return t_last_cuda_error; }

int lmrs_read_device_error(int* out_flags) {
  if (!out_flags) return LMRS_ERR_NULL;
  int rc = check_device(nullptr);
  if (rc) return rc;
  uint32_t v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, lmrs::g_device_error, sizeof(v));
  if (e != cudaSuccess) return record(e);
  e = cudaMemcpyToSymbol(lmrs::g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return record(e);
  *out_flags = static_cast<int>(v);
  return LMRS_OK;
}

// Tuning knobs for measurement sweeps; returns 0 on a known key.
int lmrs_set_tuning(const char* key, int value) {
  if (!key) return LMRS_ERR_NULL;
  if (!strcmp(key, "awq_gemv_max_m")) g_tune.awq_gemv_max_m = value;
  else if (!strcmp(key, "awq_swap_max_m")) g_tune.awq_swap_max_m = value;
  else if (!strcmp(key, "awq_swap_deep_k")) g_tune.awq_swap_deep_k = value;
  else if (!strcmp(key, "awq_swap_cluster")) g_tune.awq_swap_cluster = value;
  else if (!strcmp(key, "awq_swap_narrow_tiles")) g_tune.awq_swap_narrow_tiles = value;
  else if (!strcmp(key, "awq_gemm_pair")) g_tune.awq_gemm_pair = value;
  else if (!strcmp(key, "gemm_bn")) g_tune.gemm_bn = value;
  else if (!strcmp(key, "fp8_gemv_max_m")) g_tune.fp8_gemv_max_m = value;
  else if (!strcmp(key, "gemv_ctas_per_sm")) g_tune.gemv_ctas_per_sm = value;
  else if (!strcmp(key, "awq_gemv_cluster")) g_tune.awq_gemv_cluster = value;
  else if (!strcmp(key, "pdl")) g_tune.pdl = value ? 1 : 0;
  else if (!strcmp(key, "awq_gemv_slots")) g_tune.awq_gemv_slots = value;
  else if (!strcmp(key, "awq_gemv4")) g_tune.awq_gemv4 = value ? 1 : 0;
  else if (!strcmp(key, "gemv_box_rows")) g_tune.gemv_box_rows = value;
  else if (!strcmp(key, "awq_gemv4_slots")) g_tune.awq_gemv4_slots = value;
  else if (!strcmp(key, "attn_stages")) g_tune.attn_stages = value;
  else if (!strcmp(key, "attn_ctas_per_sm")) g_tune.attn_ctas_per_sm = value;
  else if (!strcmp(key, "attn_global_merge")) g_tune.attn_global_merge = value ? 1 : 0;
  else if (!strcmp(key, "attn_multi_min_ctx")) g_tune.attn_multi_min_ctx = value;
  else if (!strcmp(key, "fp8_gemv_cluster")) g_tune.fp8_gemv_cluster = value;
  else if (!strcmp(key, "ar_two_stage_min_world")) g_tune.ar_two_stage_min_world = value;
  else if (!strcmp(key, "ar_two_stage_min_elems")) g_tune.ar_two_stage_min_elems = value;
  else if (!strcmp(key, "fp8_gemm_group_m")) g_tune.fp8_gemm_group_m = value;
  else if (!strcmp(key, "fp8_gemm_bn128")) g_tune.fp8_gemm_bn128 = value ? 1 : 0;
  else if (!strcmp(key, "fp8_gemm_pair")) g_tune.fp8_gemm_pair = value ? 1 : 0;
  else if (!strcmp(key, "fp8_gemm_pair_min_m")) g_tune.fp8_gemm_pair_min_m = value;
  else if (!strcmp(key, "fp8_gemm_pair_ksub")) g_tune.fp8_gemm_pair_ksub = value == 2 ? 2 : 1;
  else if (!strcmp(key, "fp8_swap_max_m")) g_tune.fp8_swap_max_m = value;
  else if (!strcmp(key, "fp8_gemv_max_kn")) g_tune.fp8_gemv_max_kn = value;
  else if (!strcmp(key, "awq_tmem_max_m")) g_tune.awq_tmem_max_m = value;
  else if (!strcmp(key, "awq_gemm_tmem")) g_tune.awq_gemm_tmem = value ? 1 : 0;
  else if (!strcmp(key, "awq_gemm_tmem_bt")) g_tune.awq_gemm_tmem_bt = value;
  else if (!strcmp(key, "awq_gemm_tmem_pair")) g_tune.awq_gemm_tmem_pair = value ? 1 : 0;
  else if (!strcmp(key, "awq_gemm_tmem_bk")) g_tune.awq_gemm_tmem_bk = value;
  else if (!strcmp(key, "awq_tmem_min_m")) g_tune.awq_tmem_min_m = value;
  else if (!strcmp(key, "awq_tmem_min_m_wide")) g_tune.awq_tmem_min_m_wide = value;
  else if (!strcmp(key, "awq_tmem_cluster")) g_tune.awq_tmem_cluster = value;
  else if (!strcmp(key, "awq_tmem_ctas_per_sm")) g_tune.awq_tmem_ctas_per_sm = value;
  else if (!strcmp(key, "fp8_swap_cluster")) g_tune.fp8_swap_cluster = value;
  else if (!strcmp(key, "fp8_swap_deep_k")) g_tune.fp8_swap_deep_k = value;
  else if (!strcmp(key, "awq_i8_max_m")) g_tune.awq_i8_max_m = value;
  else if (!strcmp(key, "awq_i8_slots")) g_tune.awq_i8_slots = value;
  else if (!strcmp(key, "awq_i8_ctas_per_sm")) g_tune.awq_i8_ctas_per_sm = value;
  else if (!strcmp(key, "awq_i8_cluster")) g_tune.awq_i8_cluster = value;
  else if (!strcmp(key, "awq_i8_box_rows")) g_tune.awq_i8_box_rows = value;
  else if (!strcmp(key, "decode_layer_trace")) g_tune.decode_layer_trace = value;
  else if (!strcmp(key, "wait_limit_kcycles")) {
    // bounded-wait limit of the current device, in thousands of SM cycles
    // (<= 0 restores the default of ~2 s); a device variable, so set per device
    int rc = check_device(nullptr);
    if (rc) return rc;
    const long long v = value > 0 ? 1000LL * value : lmrs::kWaitLimitCycles;
    cudaError_t e = cudaMemcpyToSymbol(lmrs::g_wait_limit_cycles, &v, sizeof(v));
    if (e != cudaSuccess) return record(e);
  }
  else return LMRS_ERR_SHAPE;
  return LMRS_OK;
}

int lmrs_awq_unpack(int8_t* q_out, const int32_t* packed, int rows, int cols,
                    lmrs_stream_t stream) {
  if (rows < 0 || cols < 0 || cols % 8) return LMRS_ERR_SHAPE;
  if (rows == 0 || cols == 0) return LMRS_OK;
  if (!q_out || !packed) return LMRS_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(q_out) & 7u) || (reinterpret_cast<uintptr_t>(packed) & 3u))
    return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  const int64_t words = int64_t(rows) * (cols / 8);
  const int64_t blocks = (words + 255) / 256;
  lmrs::awq_unpack_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(
      q_out, reinterpret_cast<const uint32_t*>(packed), words);
  return after_launch();
}

int lmrs_awq_dequant(void* w_out, const int32_t* qweight, const int32_t* qzeros,
                     const void* scales, int K, int N, int group, lmrs_stream_t stream) {
  if (K < 0 || N < 0 || N % 8) return LMRS_ERR_SHAPE;
  if (group <= 0 || K % group) return LMRS_ERR_GROUP;
  if (K == 0 || N == 0) return LMRS_OK;
  if (!w_out || !qweight || !qzeros || !scales) return LMRS_ERR_NULL;
  if (!aligned16(w_out) || !aligned16(scales) || (reinterpret_cast<uintptr_t>(qweight) & 3u) ||
      (reinterpret_cast<uintptr_t>(qzeros) & 3u))
    return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  const int64_t words = int64_t(K) * (N / 8);
  lmrs::awq_dequant_kernel<__half><<<static_cast<unsigned>((words + 255) / 256), 256, 0,
                                     reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(w_out), reinterpret_cast<const uint32_t*>(qweight),
      reinterpret_cast<const uint32_t*>(qzeros), static_cast<const __half*>(scales), K, N / 8,
      group);
  return after_launch();
}

int lmrs_awq_dequant_dtype(void* w_out, const int32_t* qweight, const int32_t* qzeros,
                           const void* scales, int K, int N, int group, int out_dtype,
                           lmrs_stream_t stream) {
  if (out_dtype == LMRS_DTYPE_F16)
    return lmrs_awq_dequant(w_out, qweight, qzeros, scales, K, N, group, stream);
  if (out_dtype != LMRS_DTYPE_BF16) return LMRS_ERR_DTYPE;
  if (K < 0 || N < 0 || N % 8) return LMRS_ERR_SHAPE;
  if (group <= 0 || K % group) return LMRS_ERR_GROUP;
  if (K == 0 || N == 0) return LMRS_OK;
  if (!w_out || !qweight || !qzeros || !scales) return LMRS_ERR_NULL;
  if (!aligned16(w_out) || !aligned16(scales) || (reinterpret_cast<uintptr_t>(qweight) & 3u) ||
      (reinterpret_cast<uintptr_t>(qzeros) & 3u))
    return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  const int64_t words = int64_t(K) * (N / 8);
  lmrs::awq_dequant_kernel<__nv_bfloat16><<<static_cast<unsigned>((words + 255) / 256), 256, 0,
                                            reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(w_out), reinterpret_cast<const uint32_t*>(qweight),
      reinterpret_cast<const uint32_t*>(qzeros), static_cast<const __half*>(scales), K, N / 8,
      group);
  return after_launch();
}

size_t lmrs_awq_linear_workspace_bytes(int M, int K, int N, int group) {
  (void)M; (void)K; (void)N; (void)group;
  return 0;
}

int lmrs_awq_linear(void* y, const void* x, const int32_t* qweight, const int32_t* qzeros,
                    const void* scales, const void* bias_or_null, int M, int K, int N, int group,
                    int act_dtype, void* workspace, size_t workspace_bytes,
                    lmrs_stream_t stream) {
  (void)workspace; (void)workspace_bytes;
  if (act_dtype != LMRS_DTYPE_F16 && act_dtype != LMRS_DTYPE_BF16) return LMRS_ERR_DTYPE;
  if (M < 0 || K <= 0 || N <= 0 || N % 32) return LMRS_ERR_SHAPE;
  if (group <= 0 || group % 64 || K % group) return LMRS_ERR_GROUP;
  if (M == 0) return LMRS_OK;
  if (!y || !x || !qweight || !qzeros || !scales) return LMRS_ERR_NULL;
  if (!aligned16(y) || !aligned16(x) || !aligned16(qweight) || !aligned16(qzeros) ||
      !aligned16(scales) || (bias_or_null && !aligned16(bias_or_null)))
    return LMRS_ERR_ALIGN;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto* sh = static_cast<const __half*>(scales);
  if (act_dtype == LMRS_DTYPE_BF16)
    return awq_linear_dispatch<__nv_bfloat16>(
        static_cast<__nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(x), qweight, qzeros, sh,
        static_cast<const __nv_bfloat16*>(bias_or_null), M, K, N, group, st, dev);
  return awq_linear_dispatch<__half>(static_cast<__half*>(y), static_cast<const __half*>(x),
                                     qweight, qzeros, sh, static_cast<const __half*>(bias_or_null),
                                     M, K, N, group, st, dev);
}

int lmrs_fp8_quant_rows(uint8_t* q, float* scale, const void* x, int rows, int K, int x_dtype,
                        lmrs_stream_t stream) {
  if (x_dtype < 0 || x_dtype > 2) return LMRS_ERR_DTYPE;
  if (rows < 0 || K <= 0 || K % 16) return LMRS_ERR_SHAPE;
  if (rows == 0) return LMRS_OK;
  if (!q || !scale || !x) return LMRS_ERR_NULL;
  if (!aligned16(q) || !aligned16(x) || (reinterpret_cast<uintptr_t>(scale) & 3u))
    return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  return fp8_quant_launch(q, scale, x, rows, K, x_dtype, reinterpret_cast<cudaStream_t>(stream));
}

size_t lmrs_fp8_linear_workspace_bytes(int M, int K, int N) {
  (void)N;
  if (M <= 0 || K <= 0) return 0;
  return round_up(size_t(M) * size_t(K), 256) + round_up(size_t(M) * 4, 256);
}

int lmrs_fp8_linear_prequant(void* y, const uint8_t* xq, const float* x_scale, const uint8_t* wq,
                             const float* w_scale, const void* bias_or_null, int M, int K, int N,
                             lmrs_stream_t stream) {
  if (M < 0 || K <= 0 || N <= 0 || K % 16) return LMRS_ERR_SHAPE;
  if (M == 0) return LMRS_OK;
  if (!y || !xq || !x_scale || !wq || !w_scale) return LMRS_ERR_NULL;
  if (!aligned16(xq) || !aligned16(wq) || (reinterpret_cast<uintptr_t>(y) & 3u) ||
      (reinterpret_cast<uintptr_t>(x_scale) & 3u) || (reinterpret_cast<uintptr_t>(w_scale) & 3u) ||
      (reinterpret_cast<uintptr_t>(bias_or_null) & 1u))
    return LMRS_ERR_ALIGN;
  if (N % 8 && fp8_uses_gemm(M, K, N)) return LMRS_ERR_SHAPE;  // GEMM epilogue stores
  int dev = 0;
  int rc = check_device(&dev);
  if (rc) return rc;
  return fp8_linear_prequant_impl(y, xq, x_scale, wq, w_scale, bias_or_null, M, K, N,
                                  reinterpret_cast<cudaStream_t>(stream), dev);
}

int lmrs_fp8_linear(void* y, const void* x, const uint8_t* wq, const float* w_scale,
                    const void* bias_or_null, int M, int K, int N, void* workspace,
                    size_t workspace_bytes, lmrs_stream_t stream) {
  if (M < 0 || K <= 0 || N <= 0 || K % 16) return LMRS_ERR_SHAPE;
  if (M == 0) return LMRS_OK;
  if (!y || !x || !wq || !w_scale) return LMRS_ERR_NULL;
  const size_t need = lmrs_fp8_linear_workspace_bytes(M, K, N);
  if (!workspace || workspace_bytes < need) return LMRS_ERR_WORKSPACE;
  if (!aligned16(workspace) || !aligned16(x) || !aligned16(wq) ||
      (reinterpret_cast<uintptr_t>(y) & 3u) || (reinterpret_cast<uintptr_t>(w_scale) & 3u) ||
      (reinterpret_cast<uintptr_t>(bias_or_null) & 1u))
    return LMRS_ERR_ALIGN;
  if (N % 8 && fp8_uses_gemm(M, K, N)) return LMRS_ERR_SHAPE;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* xq = static_cast<uint8_t*>(workspace);
  float* sx = reinterpret_cast<float*>(xq + round_up(size_t(M) * size_t(K), 256));
  if ((rc = fp8_quant_launch(xq, sx, x, M, K, LMRS_DTYPE_BF16, st))) return rc;
  return fp8_linear_prequant_impl(y, xq, sx, wq, w_scale, bias_or_null, M, K, N, st, dev);
}

}  // extern "C"

// ======================================== FP8 linear with library-held scratch
// For callers that cannot allocate device memory (see lmrs_quant.h).  The
// scratch is a file-scope device array; in host code its name is only a
// host-side stand-in, so the device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and passed to the kernels.
static __device__ __align__(256) uint8_t lmrs_fp8_noalloc_scratch[LMRS_FP8_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices];  // device address per device, nullptr until looked up

int noalloc_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, lmrs_fp8_noalloc_scratch);
    if (e != cudaSuccess) return record(e);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LMRS_OK;
}
}  // namespace

extern "C" int lmrs_fp8_linear_noalloc(void* y, const void* x, const uint8_t* wq,
                                       const float* w_scale, const void* bias_or_null, int M,
                                       int K, int N, lmrs_stream_t stream) {
  if (M < 0 || K <= 0 || N <= 0 || K % 16) return LMRS_ERR_SHAPE;
  if (M == 0) return LMRS_OK;
  if (!y || !x || !wq || !w_scale) return LMRS_ERR_NULL;
  if (lmrs_fp8_linear_workspace_bytes(M, K, N) > LMRS_FP8_NOALLOC_SCRATCH_BYTES)
    return LMRS_ERR_TOO_LARGE;
  if (!aligned16(x) || !aligned16(wq) || (reinterpret_cast<uintptr_t>(y) & 3u) ||
      (reinterpret_cast<uintptr_t>(w_scale) & 3u) ||
      (reinterpret_cast<uintptr_t>(bias_or_null) & 1u))
    return LMRS_ERR_ALIGN;
  if (N % 8 && fp8_uses_gemm(M, K, N)) return LMRS_ERR_SHAPE;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc) return rc;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(dev, &scratch))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* xq = static_cast<uint8_t*>(scratch);
  float* sx = reinterpret_cast<float*>(xq + round_up(size_t(M) * size_t(K), 256));
  if ((rc = fp8_quant_launch(xq, sx, x, M, K, LMRS_DTYPE_BF16, st))) return rc;
  return fp8_linear_prequant_impl(y, xq, sx, wq, w_scale, bias_or_null, M, K, N, st, dev);
}

// decode-step kernels around the quantized linears (include/lmrs_decode.h)
#include "decode_capi.cuh"

// tensor-parallel all-reduce (include/lmrs_comm.h)
#include "comm_capi.cuh"

// persistent FP8 decode layer (include/lmrs_layer.h; uses the all-reduce buffers above)
#include "decode_layer_capi.cuh"
