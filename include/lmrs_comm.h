/*
 * lmrs_comm.h — C-ABI of the tensor-parallel all-reduce that follows the
 * row-parallel quantized projections (o and down) of a decode step.
 *
 * The reference reduces across GPUs with its custom all-reduce over IPC-mapped
 * buffers (kernels/comm/custom_all_reduce.cuh, signal flags + one/two-shot
 * kernels).  This one-shot version moves the flag into each 8-byte packet
 * beside 4 bytes of data (see lmrs_b200/csrc/allreduce.cuh), so a call is one
 * kernel with no barrier round trip.  The caller owns the buffers; the IPC
 * helpers below let a host runtime share them between the processes of one
 * node (one process per GPU), the way the reference's Rust side wires its
 * custom all-reduce handles.
 */
#ifndef LMRS_COMM_H
#define LMRS_COMM_H

#include "lmrs_quant.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Bytes of one rank's receive buffer for `world` ranks and vectors of up to
 * max_elems 16-bit elements (max_elems even). */
LMRS_API size_t lmrs_allreduce_buffer_bytes(int world, size_t max_elems);

/* Device allocation (the current device), zero-filled; its own IPC base. */
LMRS_API int lmrs_comm_alloc(void** ptr_out, size_t bytes);
LMRS_API int lmrs_comm_free(void* ptr);

/* cudaIpcMemHandle of an lmrs_comm_alloc pointer (handle_bytes >= 64), and the
 * peer side: map / unmap a handle received from another process. */
LMRS_API int lmrs_ipc_get_handle(void* ptr, void* handle_out, size_t handle_bytes);
LMRS_API int lmrs_ipc_open(const void* handle, void** ptr_out);
LMRS_API int lmrs_ipc_close(void* ptr);

/* out = sum over the `world` ranks of in (n elements, n even, n <= max_elems;
 * dtype bf16 or f16; out may equal in).  buffers: host array of the world
 * receive buffers (lmrs_comm_alloc of lmrs_allreduce_buffer_bytes(world,
 * max_elems) bytes each, peers' mapped through lmrs_ipc_open), in rank order.
 * Every rank must issue the same sequence of calls (same n) on its stream;
 * results are bit-identical on all ranks.  A wait for a peer that never
 * arrives gives up after ~2 s (lmrs_set_tuning "wait_limit_kcycles"), flags
 * kErrWaitPeer (bit 5) in lmrs_read_device_error and leaves NaN in every
 * output element that source's packets did not reach.  From 4 ranks and 131072
 * elements (lmrs_set_tuning "ar_two_stage_min_world" / "ar_two_stage_min_elems")
 * the sum runs as reduce-scatter + all-gather in one kernel (about 2n packets
 * per rank instead of world x n), with the same result. */
LMRS_API int lmrs_allreduce_sum(void* out, const void* in, size_t n, int dtype, int rank,
                                int world, void* const* buffers, size_t max_elems,
                                lmrs_stream_t stream);

/* The all-reduce of a row-parallel projection fused with the residual add and
 * RMSNorm that follow it (one launch instead of lmrs_allreduce_sum then
 * lmrs_rmsnorm[_fp8]): for rows x H elements (H % 8 == 0, H <= 32768,
 * rows * H <= max_elems),
 *   delta    = sum over ranks of partial (rank order in fp32, rounded once to
 *              dtype: the same values lmrs_allreduce_sum produces),
 *   residual = dtype(residual + delta)        (in place),
 *   out      = rmsnorm(residual) * weight     (one rounding),
 * the _fp8 form writing the e4m3 bytes and per-row scale of that output
 * instead (as lmrs_fp8_quant_rows of it).  partial is read only.  Same buffers,
 * call-order and bounded-wait rules as lmrs_allreduce_sum (the two share the
 * buffers' epoch, so calls of both may alternate); world may be 1.  All
 * pointers 16-byte aligned.  Replaces, on the decode step's data path, the
 * reference's custom all-reduce (kernels/comm/custom_all_reduce.cuh) followed
 * by rmsnorm_fwd (kernels/ffi/norm_ffi.cu:87-95). */
LMRS_API int lmrs_allreduce_rmsnorm(void* out, void* residual, const void* partial,
                                    const void* weight, int rows, int H, float eps, int dtype,
                                    int rank, int world, void* const* buffers, size_t max_elems,
                                    lmrs_stream_t stream);
LMRS_API int lmrs_allreduce_rmsnorm_fp8(uint8_t* q_out, float* scale_out, void* residual,
                                        const void* partial, const void* weight, int rows, int H,
                                        float eps, int dtype, int rank, int world,
                                        void* const* buffers, size_t max_elems,
                                        lmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LMRS_COMM_H */
