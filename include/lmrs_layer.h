/*
 * lmrs_layer.h — C-ABI of the persistent FP8 decode-layer kernel (B200, sm_100a):
 * one launch runs a whole decoder layer of a W8A8 decode step (residual add +
 * RMSNorm, merged q/k/v projection, RoPE + KV write, paged GQA attention, o
 * projection, its all-reduce, residual add + RMSNorm, merged gate/up, SiLU * up,
 * down projection and its all-reduce) for up to 8 tokens.
 *
 * It fuses, for one layer, what the reference's block forward does with
 * separate calls (crates/model/src/layers/block.rs:118-130: rmsnorm_fwd,
 * linear_fwd x 4 through kernels/ffi/tensor_ffi.cu:820-841 with the FP8 W8A8
 * operands of lmrs_fp8_linear_prequant, pos_embed, paged_attention_v1_fwd,
 * silu_mul) plus the tensor-parallel all-reduce of lmrs_allreduce_sum; each
 * step keeps the semantics of the entry point in lmrs_quant.h / lmrs_decode.h /
 * lmrs_comm.h that it replaces (projections agree with them within fp32
 * accumulation order, not bit for bit).
 *
 * Same conventions as lmrs_quant.h: plain pointers, caller-owned buffers,
 * stream-ordered, int status, nothing launched on a rejected argument.
 * Activations, norm weights, cos/sin and the KV cache are bf16.
 */
#ifndef LMRS_LAYER_H
#define LMRS_LAYER_H

#include "lmrs_quant.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One layer's weights (this rank's shards), all device pointers, 16-byte
 * aligned.  Projections are e4m3 [N, K] row-major with fp32 per-output-channel
 * scales (lmrs_fp8_linear's weight layout):
 *   qkv      N = (num_heads + 2 num_kv_heads) * head_size, K = hidden (q | k | v)
 *   o        N = hidden, K = num_heads * head_size
 *   gate_up  N = 2 intermediate, K = hidden (gate | up)
 *   down     N = hidden, K = intermediate
 * key_cache / value_cache: [blocks][num_kv_heads][block_size][head_size]
 * (paged_attention_v1's layout, as lmrs_paged_attention_decode). */
typedef struct lmrs_fp8_layer {
  const uint8_t* qkv_weight;
  const float* qkv_scale;
  const uint8_t* o_weight;
  const float* o_scale;
  const uint8_t* gate_up_weight;
  const float* gate_up_scale;
  const uint8_t* down_weight;
  const float* down_scale;
  const void* input_norm;   /* [hidden] */
  const void* post_norm;    /* [hidden] */
  void* key_cache;
  void* value_cache;
} lmrs_fp8_layer_t;

/* Shapes of one rank's layer.  num_seqs 1..8 (one decode token per sequence),
 * head_size 128, num_heads / num_kv_heads <= 8, hidden and intermediate and
 * num_heads * head_size multiples of 128; num_seqs * (largest K + 16) <= 96 KB
 * (the quantised row of every token is held in shared memory). */
typedef struct lmrs_fp8_layer_shape {
  int num_seqs;
  int hidden;
  int num_heads;
  int num_kv_heads;
  int head_size;
  int intermediate;
  int block_size;
  int max_blocks_per_seq;
  int max_context;      /* upper bound of context_lens: sizes the attention chunks */
  float eps;            /* RMSNorm epsilon */
  float scale;          /* attention softmax scale */
} lmrs_fp8_layer_shape_t;

/* Flags of lmrs_fp8_decode_layer (tensor parallel, world > 1). */
#define LMRS_LAYER_RECV_DELTA 1  /* residual += all-reduce of the previous layer's down output */
#define LMRS_LAYER_PUSH_DELTA 2  /* push this layer's down output for the next layer's launch */

/* Bytes of the workspace for these shapes on the current device (barrier
 * words, work schedule, per-CTA statistics, intermediate rows, attention
 * partials); 0 when the shapes are not supported. */
LMRS_API size_t lmrs_fp8_decode_layer_workspace_bytes(const lmrs_fp8_layer_shape_t* shape);

/* Set a workspace up for these shapes on the current device: zeroes the
 * barrier words and writes the schedule that assigns the projections' 16-row
 * weight units to the CTAs (balanced by cumulative weight bytes).  Synchronises
 * `stream`; call once after allocating the workspace (not during stream
 * capture), and again after a call that reported LMRS_ERR_TIMEOUT. */
LMRS_API int lmrs_fp8_decode_layer_prepare(const lmrs_fp8_layer_shape_t* shape, void* workspace,
                                           size_t workspace_bytes, lmrs_stream_t stream);

/* One decoder layer for num_seqs tokens (position context_lens[s] - 1 of each
 * sequence; its k and v are written into the cache):
 *   residual (+)= delta                      delta: the previous layer's down
 *                                            output: delta_in (one rank, NULL =
 *                                            none) or, with RECV_DELTA, its
 *                                            all-reduce over the ranks
 *   x = rmsnorm(residual) * input_norm; qkv = x W_qkv^T (per-token e4m3)
 *   RoPE(q, k) with cos / sin [head_size / 2]; k, v -> cache
 *   a = softmax(scale q k^T) v per q head (KV head h / (num_heads / num_kv_heads))
 *   residual += allreduce(a W_o^T)
 *   x = rmsnorm(residual) * post_norm; gu = x W_gate_up^T
 *   d = (silu(gate) * up) W_down^T  -> delta_out (bf16 [num_seqs, hidden]) unless
 *                                     PUSH_DELTA, which pushes it to the ranks
 *                                     for the next layer's RECV_DELTA instead
 * residual: bf16 [num_seqs, hidden], updated in place.  world 1: rank 0,
 * buffers NULL.  world 2..8: buffers / max_elems of lmrs_allreduce_sum (the
 * same call-order rule: every rank makes the same calls in the same order;
 * this call takes part in 1 + (RECV_DELTA) + (PUSH_DELTA) of its all-reduce
 * calls), max_elems >= num_seqs * hidden.  The last layer leaves PUSH_DELTA
 * off and hands delta_out to lmrs_allreduce_rmsnorm for the final norm.
 * One CTA per SM, launched cooperatively (all resident); calls that overlap on
 * the GPU need separate workspaces.  A bounded wait that gave up sets the
 * device error word (lmrs_read_device_error); prepare the workspace again. */
LMRS_API int lmrs_fp8_decode_layer(const lmrs_fp8_layer_t* layer,
                                   const lmrs_fp8_layer_shape_t* shape, void* residual,
                                   const void* delta_in_or_null, void* delta_out, int flags,
                                   const int32_t* block_tables, const int32_t* context_lens,
                                   const void* cos, const void* sin, int rank, int world,
                                   void* const* buffers, size_t max_elems, void* workspace,
                                   size_t workspace_bytes, lmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LMRS_LAYER_H */
