/*
 * lmrs_quant.h — C-ABI of the B200 (sm_100a) quantized-linear kernels.
 *
 * Drop-in boundary for lmrs's linear hot path.  The reference exposes one dense
 * linear entry point, `extern "C" void linear_fwd(out, input, weight, bias, rows,
 * in_features, out_features, dtype, stream)` (kernels/ffi/tensor_ffi.cu:820-841),
 * declared on the Rust side at crates/kernels/src/tensor_ops.rs:18 and called by
 * `kernels::linear` (crates/kernels/src/tensor_ops.rs:225-246) from
 * `LinearOp::forward` (crates/ops/src/linear/linear.rs:33-35).  The quantized
 * linears below join that boundary in the same style:
 *
 *   - plain pointers and sizes, no tensor types;
 *   - the caller owns every buffer (output and workspace included), exactly as
 *     `kernels::linear` allocates the output on the input's stream
 *     (crates/kernels/src/tensor_ops.rs:236-237);
 *   - the launch is stream-ordered and returns at once;
 *   - unlike `linear_fwd`, which silently ignores an unknown dtype
 *     (kernels/ffi/tensor_ffi.cu:830-840), every entry point returns an int
 *     status (LMRS_OK = 0) and launches nothing when it rejects its arguments.
 *
 * Dtype codes follow the reference's `KernelDType{Bf16=0, F16=1, F32=2}`
 * (crates/kernels/src/raw.rs:9-13).
 *
 * Formats (the reference defines neither; they are fixed by the task's configs):
 *   AWQ W4A16: qweight int32 [K, N/8]; word j of row k holds columns 8j..8j+7,
 *     nibble i (bits 4i..4i+3) = column 8j + ORDER[i], ORDER = {0,2,4,6,1,3,5,7}.
 *     qzeros int32 [K/g, N/8] packed the same way; scales fp16 [K/g, N].
 *     Activations x, y, bias are fp16 or bf16 (act_dtype); the dequantised
 *     weight has the activation type and is the exact product rounded once:
 *     w[k,n] = T_rne((q[k,n] - z[k/g,n]) * s[k/g,n]), T = fp16 or bf16;
 *     y[m,n] = T(sum_k x[m,k] * w[k,n] (+ bias[n])), fp32 accumulation.
 *   FP8 W8A8: wq e4m3 [N, K] (same [out, in] layout as LinearOp's weight,
 *     crates/ops/src/linear/linear.rs:48-66), w_scale fp32 [N];
 *     s_x[m] = absmax_k |x[m,k]| / 448, xq = e4m3_rne_satfinite(x / s_x)
 *     (rows with s_x == 0 quantize to 0);
 *     y[m,n] = bf16(acc * s_x[m] * s_w[n] (+ bias[n])), acc = sum_k xq * wq in fp32.
 */
#ifndef LMRS_QUANT_H
#define LMRS_QUANT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LMRS_API __attribute__((visibility("default")))
#else
#define LMRS_API
#endif

/* cudaStream_t without pulling in cuda_runtime.h (same ABI: a pointer). */
typedef struct CUstream_st* lmrs_stream_t;

/* ---- status codes ------------------------------------------------------- */
enum {
  LMRS_OK = 0,
  LMRS_ERR_SHAPE = 1,        /* a dimension is <= 0 or breaks a divisibility rule */
  LMRS_ERR_DTYPE = 2,        /* dtype code not supported by this entry point */
  LMRS_ERR_ALIGN = 3,        /* a pointer is not 16-byte aligned */
  LMRS_ERR_GROUP = 4,        /* group size does not divide K, or is not a multiple of 64 */
  LMRS_ERR_WORKSPACE = 5,    /* workspace missing or smaller than *_workspace_bytes */
  LMRS_ERR_CUDA = 6,         /* a CUDA runtime/driver call failed (see lmrs_last_cuda_error) */
  LMRS_ERR_DEVICE = 7,       /* current device is not sm_100 */
  LMRS_ERR_NULL = 8,         /* a required pointer is NULL */
  LMRS_ERR_TIMEOUT = 9,      /* a kernel's bounded wait gave up (lmrs_read_device_error) */
  LMRS_ERR_TOO_LARGE = 10    /* problem needs more scratch than lmrs_fp8_linear_noalloc holds */
};

enum { LMRS_DTYPE_BF16 = 0, LMRS_DTYPE_F16 = 1, LMRS_DTYPE_F32 = 2 };

/* Human-readable text for a status code (static storage). */
LMRS_API const char* lmrs_status_string(int status);
/* Last CUDA error code (cudaError_t as int) recorded by a failing entry point. */
LMRS_API int lmrs_last_cuda_error(void);
/* Reads and clears the device-side error word of the current device: nonzero
 * when a kernel's bounded mbarrier wait expired (bit layout in lmrs_ptx.cuh).
 * Synchronous (copies 4 bytes from the device). */
LMRS_API int lmrs_read_device_error(int* out_flags);
/* Library version, for the binding's sanity check. */
LMRS_API int lmrs_version(void);
/* Measurement knobs (dispatch thresholds, split-K shape, launch mode); 0 on a
 * known key, LMRS_ERR_SHAPE otherwise.  Keys: "awq_gemv_max_m", "awq_swap_max_m",
 * "awq_swap_deep_k" (swap-AB up to 128 tokens when 4K >= value x N, default 5; 0 = off),
 * "awq_swap_cluster", "awq_swap_narrow_tiles" (swap-AB up to 128 tokens while N / 128
 * is at most this, default 32; 0 = off), "awq_gemm_pair", "gemm_bn", "fp8_gemv_max_m",
 * "gemv_ctas_per_sm", "awq_gemv_cluster", "fp8_gemv_cluster", "fp8_gemv_max_kn",
 * "fp8_swap_max_m", "fp8_swap_cluster", "fp8_swap_deep_k" (decode FP8 on the swap-AB kernel
 * when K >= this x N, default 4; 0 = off), "fp8_gemm_group_m" (FP8 GEMM tile order: M
 * tiles per group, default 32), "fp8_gemm_bn128" (128-wide FP8 GEMM tiles while
 * that grid fits one wave, default 1), "fp8_gemm_pair" (CTA-pair 256 x 256 FP8 GEMM
 * tiles where the 128-wide ones exceed a wave, default 1), "fp8_gemm_pair_min_m" (... from
 * this many tokens, default 256),
 * "fp8_gemm_pair_ksub" (its K stage: 1 = 128 bytes, 2 = 256 bytes, default 2), "awq_tmem_min_m", "awq_tmem_max_m",
 * "awq_tmem_min_m_wide", "awq_tmem_cluster", "awq_tmem_ctas_per_sm", "awq_gemm_tmem",
 * "awq_gemm_tmem_bt", "awq_gemv4", "awq_gemv_slots", "awq_gemv4_slots",
 * "gemv_box_rows", "attn_stages", "attn_ctas_per_sm", "attn_global_merge" (small
 * batches split the context over several 8-CTA clusters merged through the
 * attention workspace, default 1), "attn_multi_min_ctx" (... only when
 * max_context exceeds it, default 2048), "awq_i8_max_m" (1-2 token
 * AWQ on the integer MMA path up to this M, default 1; 0 = fp16 GEMV),
 * "awq_i8_slots", "awq_i8_ctas_per_sm", "awq_i8_cluster", "awq_i8_box_rows", "pdl" (programmatic
 * dependent launch on every kernel, default 1), "ar_two_stage_min_world" /
 * "ar_two_stage_min_elems" (lmrs_allreduce_sum's two-stage form, defaults 4 /
 * 131072), "decode_layer_trace" (1: lmrs_fp8_decode_layer records global-timer
 * stamps at the start and around every grid barrier, 32 per CTA, in the last
 * grid x 256 bytes of its workspace; default 0), "wait_limit_kcycles" (how long a
 * kernel's bounded wait spins before it gives up and flags the device error
 * word, in thousands of SM cycles, on the CURRENT device only; <= 0 restores the
 * default of ~2 s; synchronous).
 * Process-wide, not thread-safe against concurrent launches: for measurement and
 * tests, not for a host's hot path. */
LMRS_API int lmrs_set_tuning(const char* key, int value);

/* ---- AWQ W4A16 ----------------------------------------------------------- */

/* Unpack AWQ-packed int4: packed int32 [rows, cols/8] -> q int8 [rows, cols],
 * column order restored (q[r, 8j + ORDER[i]] = nibble i of packed[r, j]).
 * Works for qweight (rows = K) and qzeros (rows = K/g).  cols % 8 == 0.
 * No reference counterpart: the reference has no AWQ code; this restates the
 * unpack that the orphaned kernels/moe/moe_wna16_utils.h:102-175 performs in
 * registers. */
LMRS_API int lmrs_awq_unpack(int8_t* q_out, const int32_t* packed, int rows, int cols,
                    lmrs_stream_t stream);

/* Dequantize to fp16 [K, N]: w = fp16_rne((q - z) * s), bit-exact.
 * K % group == 0, N % 8 == 0.  Replaces the weight tensor that
 * `LinearOp` would hold (crates/ops/src/linear/linear.rs:15-18), transposed. */
LMRS_API int lmrs_awq_dequant(void* w_out, const int32_t* qweight, const int32_t* qzeros,
                     const void* scales, int K, int N, int group,
                     lmrs_stream_t stream);

/* The same dequant to the activation type out_dtype: LMRS_DTYPE_F16 (as
 * lmrs_awq_dequant) or LMRS_DTYPE_BF16, w = bf16_rne((q - z) * s) with the
 * fp16 scale as stored (one rounding of the exact product), bit-exact.  These
 * are the weights the bf16 lmrs_awq_linear multiplies by (the GEMV regimes
 * apply the scale to integer sums instead and round nothing per weight). */
LMRS_API int lmrs_awq_dequant_dtype(void* w_out, const int32_t* qweight,
                                    const int32_t* qzeros, const void* scales, int K,
                                    int N, int group, int out_dtype, lmrs_stream_t stream);

/* Workspace for lmrs_awq_linear.  Returns 0: the AWQ linear keeps its split-K
 * partial sums in thread-block-cluster shared memory and needs no scratch. */
LMRS_API size_t lmrs_awq_linear_workspace_bytes(int M, int K, int N, int group);

/* y[M,N] = x[M,K] @ dequant(qweight, qzeros, scales) (+ bias[N]).
 * act_dtype is the type of x, y and bias: LMRS_DTYPE_BF16 (the reference
 * model's dtype, crates/kernels/src/raw.rs:9-13) or LMRS_DTYPE_F16; scales are
 * fp16 either way.  Requirements:
 * K % group == 0, group % 64 == 0, N % 32 == 0, 16-byte aligned pointers.
 * M <= 8 runs a register-dequant tensor-core GEMV (HBM bound); M <= 64 a
 * swap-AB split-K tcgen05 kernel; larger M a persistent tcgen05 GEMM (one SM
 * per 128x256 tile, or CTA pairs with "awq_gemm_pair").  The tcgen05 paths fuse
 * the dequant into the shared-memory stage.
 * Replaces `linear_fwd` (kernels/ffi/tensor_ffi.cu:820-841) for AWQ layers. */
LMRS_API int lmrs_awq_linear(void* y, const void* x, const int32_t* qweight,
                    const int32_t* qzeros, const void* scales,
                    const void* bias_or_null, int M, int K, int N, int group,
                    int act_dtype, void* workspace, size_t workspace_bytes,
                    lmrs_stream_t stream);

/* ---- FP8 e4m3 W8A8 -------------------------------------------------------- */

/* Per-row (per-token for activations, per-output-channel for weights) e4m3
 * quantization: scale[r] = absmax / 448, q[r, :] = e4m3(x[r, :] / scale[r]).
 * x_dtype: LMRS_DTYPE_BF16 / F16 / F32.  K % 16 == 0.
 * No reference counterpart: `CastKind::Quantized` is disallowed in the reference
 * (crates/tensor/src/dtype/cast.rs:30-45). */
LMRS_API int lmrs_fp8_quant_rows(uint8_t* q, float* scale, const void* x, int rows, int K,
                        int x_dtype, lmrs_stream_t stream);

/* Workspace for lmrs_fp8_linear: the quantized activations (M*K bytes, padded)
 * plus M fp32 scales. */
LMRS_API size_t lmrs_fp8_linear_workspace_bytes(int M, int K, int N);

/* y bf16 [M,N] = per-token-quant(x bf16 [M,K]) @ wq^T, scaled by s_x[m]*w_scale[n]
 * (+ bias bf16 [N]).  K % 16 == 0.  Replaces `linear_fwd` for FP8 layers. */
LMRS_API int lmrs_fp8_linear(void* y, const void* x, const uint8_t* wq,
                    const float* w_scale, const void* bias_or_null, int M, int K,
                    int N, void* workspace, size_t workspace_bytes,
                    lmrs_stream_t stream);

/* Same GEMM on activations that are already quantized (xq e4m3 [M,K], x_scale
 * fp32 [M]), e.g. by a fused norm->quant kernel. */
LMRS_API int lmrs_fp8_linear_prequant(void* y, const uint8_t* xq, const float* x_scale,
                             const uint8_t* wq, const float* w_scale,
                             const void* bias_or_null, int M, int K, int N,
                             lmrs_stream_t stream);

/* ---- FP8 W8A8 without any device allocation -------------------------------
 * No counterpart in the reference: lmrs's `kernels::linear` always allocates
 * its output on the stream (crates/kernels/src/tensor_ops.rs:236-237) and has
 * no scratch; this entry point exists for callers that cannot allocate.
 *
 * Same result as lmrs_fp8_linear (same kernels), but the quantised activations
 * live in a scratch array compiled into this library: a file-scope
 * `static __device__` array of LMRS_FP8_NOALLOC_SCRATCH_BYTES, which every GPU
 * that loads the library holds until the process exits.  For callers that
 * cannot call cudaMalloc or any allocator at the point of the call — a host
 * runtime whose device memory is owned by its own pool with no hook for a
 * plugin's scratch, a decode loop that must not allocate after warm-up, a
 * process that must keep its device footprint fixed after load.  The caller
 * still owns and passes x, wq, w_scale, bias and y.
 *
 *   - Limit: lmrs_fp8_linear_workspace_bytes(M, K, N) must not exceed
 *     LMRS_FP8_NOALLOC_SCRATCH_BYTES (4 MiB: e.g. M*K up to about 4.1 million
 *     e4m3 bytes — M=256 at K=14336, M=1024 at K=4096); larger problems return
 *     LMRS_ERR_TOO_LARGE and launch nothing.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture.
 *   - Every call on a device shares the one array and leaves its contents
 *     behind; nothing in it needs to start at zero (each call overwrites the
 *     bytes it reads).  Calls that overlap on the GPU — on two streams, or from
 *     two threads — race on the array: serialise them.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
#define LMRS_FP8_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)
LMRS_API int lmrs_fp8_linear_noalloc(void* y, const void* x, const uint8_t* wq,
                                     const float* w_scale, const void* bias_or_null, int M,
                                     int K, int N, lmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LMRS_QUANT_H */
