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
 * output element that source's packets did not reach. */
LMRS_API int lmrs_allreduce_sum(void* out, const void* in, size_t n, int dtype, int rank,
                                int world, void* const* buffers, size_t max_elems,
                                lmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LMRS_COMM_H */
