/*
 * lmrs_decode.h — C-ABI of the B200 (sm_100a) kernels around the quantized
 * linears in a decode step: the path's edges (norm -> quantized linear,
 * activation -> quantized linear) and the decode attention between q/k/v and o.
 *
 * Same conventions as lmrs_quant.h (plain pointers, caller-owned buffers,
 * stream-ordered, int status, nothing launched on a rejected argument, dtype
 * codes LMRS_DTYPE_BF16 / LMRS_DTYPE_F16).  Each entry point names the
 * reference FFI function whose semantics it keeps.
 */
#ifndef LMRS_DECODE_H
#define LMRS_DECODE_H

#include "lmrs_quant.h"

#ifdef __cplusplus
extern "C" {
#endif

/* RMSNorm over rows of H (H % 8 == 0, H <= 32768: a row is held in one CTA's
 * registers), optionally fused with the residual add:
 *   if delta: residual[r] = round(residual[r] + delta[r])   (in place)
 *   out[r, c] = round(residual[r, c] * rsqrt(mean_c residual[r]^2 + eps) * weight[c])
 * The normalisation is the reference's rmsnorm_fwd (kernels/ffi/norm_ffi.cu:9-31,
 * 87-95: fp32 math, one rounding); the residual add replaces a separate binary
 * add kernel.  dtype: bf16 or f16. */
LMRS_API int lmrs_rmsnorm(void* out, void* residual, const void* delta_or_null,
                          const void* weight, int rows, int H, float eps, int dtype,
                          lmrs_stream_t stream);

/* Same, but the normalised rows leave as FP8 W8A8 activations: e4m3 bytes
 * q_out[rows, H] and per-row scales scale_out[rows], bit-identical to
 * lmrs_rmsnorm followed by lmrs_fp8_quant_rows; feeds lmrs_fp8_linear_prequant. */
LMRS_API int lmrs_rmsnorm_fp8(uint8_t* q_out, float* scale_out, void* residual,
                              const void* delta_or_null, const void* weight, int rows, int H,
                              float eps, int dtype, lmrs_stream_t stream);

/* out[r, i] = round(silu(gate_up[r, i]) * gate_up[r, inter + i]) for a merged
 * gate|up projection output [rows, 2 * inter] (inter % 8 == 0); silu(x) =
 * x / (1 + exp(-x)) as the reference's silu_mul (kernels/ops/activation_kernels.cuh:40-48). */
LMRS_API int lmrs_silu_mul(void* out, const void* gate_up, int rows, int inter, int dtype,
                           lmrs_stream_t stream);

/* Same, leaving as FP8 activations (bytes [rows, inter] + per-row scales);
 * inter <= 65536 (rows wider than 8192 are split over a thread-block cluster
 * whose CTAs exchange the row absmax through distributed shared memory). */
LMRS_API int lmrs_silu_mul_fp8(uint8_t* q_out, float* scale_out, const void* gate_up, int rows,
                               int inter, int dtype, lmrs_stream_t stream);

/* Rotate-half RoPE of the q and k heads of a merged qkv row
 * [num_seqs, (num_heads + 2 * num_kv_heads) * head_size] at each sequence's
 * position positions[s], as the reference's rope_fwd (kernels/ffi/pos_embed_ffi.cu:9-29,
 * cos/sin given for that position: head_size / 2 entries each):
 *   q_out[s, h, :] = rope(q);  k/v written into the paged cache at positions[s]
 *   (cache[block][kv_head][block_offset][head_size], block = block_tables[s,
 *   positions[s] / block_size], as paged_attention_v1 reads it).  head_size even
 *   (16-byte vector path when head_size % 16 == 0 and every pointer is 16-byte
 *   aligned). */
LMRS_API int lmrs_rope_kv_write(void* q_out, void* key_cache, void* value_cache,
                                const void* qkv, const void* cos, const void* sin,
                                const int32_t* block_tables, const int32_t* positions,
                                int num_seqs, int num_heads, int num_kv_heads, int head_size,
                                int block_size, int max_blocks_per_seq, int dtype,
                                lmrs_stream_t stream);

/* Workspace for lmrs_paged_attention_decode with these sizes on the current
 * device: 0 when the context splits of each sequence and KV head are few enough
 * (<= 8) to merge their partials in a thread-block cluster's distributed shared
 * memory; otherwise (small batches, contexts above 2048) room for the fp32
 * (O, m, l) partial of every 8-split cluster plus one arrival counter per
 * sequence and KV head.
 * The workspace must be zero-filled before its first use; every call leaves
 * the counters at zero again.  Calls that overlap on the GPU need separate
 * workspaces. */
LMRS_API size_t lmrs_paged_attention_workspace_bytes(int num_seqs, int num_heads,
                                                     int num_kv_heads, int max_context);

/* One decode query per sequence against a paged KV cache: the arguments of the
 * reference's paged_attention_v1_fwd (kernels/ffi/attention_ffi.cu:8-40, layout
 * and masking of kernels/attention/paged_attention.cuh:14-108) plus
 *   max_context   an upper bound of context_lens (sizes the context split),
 *   kv_head_map   0: q head h reads KV head h % num_kv_heads (the reference's
 *                 kernel), 1: h / (num_heads / num_kv_heads) (grouped heads),
 *   workspace     lmrs_paged_attention_workspace_bytes() bytes, 16-byte aligned,
 *                 zero-filled before first use (NULL when that size is 0);
 *                 LMRS_ERR_WORKSPACE if missing or smaller.
 * head_size must be 128; num_heads / num_kv_heads <= 16.  out[s, h, :] =
 * softmax(scale * q . k) v over positions [0, context_lens[s]); context 0 gives 0. */
LMRS_API int lmrs_paged_attention_decode(void* out, const void* query, const void* key_cache,
                                         const void* value_cache, const int32_t* block_tables,
                                         const int32_t* context_lens, int num_seqs, int num_heads,
                                         int num_kv_heads, int head_size, int block_size,
                                         int max_blocks_per_seq, int max_context, float scale,
                                         int kv_head_map, int dtype, void* workspace,
                                         size_t workspace_bytes, lmrs_stream_t stream);

/* lmrs_paged_attention_decode followed by lmrs_fp8_quant_rows of its output rows
 * ([num_seqs, num_heads * head_size] -> e4m3 q_out, fp32 scale_out[num_seqs]):
 * the input of an FP8 o projection.  With one KV head (a tensor-parallel rank
 * holding one KV head) the attention's final merge quantises whole rows itself
 * (one launch); otherwise two launches.  Bytes and scales equal the two calls
 * made separately; out is written as well.  q_out 16-byte aligned. */
LMRS_API int lmrs_paged_attention_decode_fp8(uint8_t* q_out, float* scale_out, void* out,
                                             const void* query, const void* key_cache,
                                             const void* value_cache, const int32_t* block_tables,
                                             const int32_t* context_lens, int num_seqs,
                                             int num_heads, int num_kv_heads, int head_size,
                                             int block_size, int max_blocks_per_seq,
                                             int max_context, float scale, int kv_head_map,
                                             int dtype, void* workspace, size_t workspace_bytes,
                                             lmrs_stream_t stream);

/* lmrs_rope_kv_write with positions = context_lens - 1 followed by
 * lmrs_paged_attention_decode (or its _fp8 form when q_out_or_null is given), in
 * one launch: qkv is the merged projection row [num_seqs, (num_heads +
 * 2 num_kv_heads) * head_size]; each CTA rotates its q heads in registers and the
 * one whose context split holds the new token rotates its k and writes k and v
 * into the cache before reading it.  Same bits as the separate calls (out,
 * cache, and the e4m3 bytes / scales); the rotated q is not written out.  cos,
 * sin: [head_size / 2] in dtype, 16-byte aligned.  With an FP8 output and more
 * than one KV head the row quantisation is a second launch. */
LMRS_API int lmrs_rope_paged_attention_decode(
    void* out, uint8_t* q_out_or_null, float* scale_out_or_null, const void* qkv,
    const void* cos, const void* sin, void* key_cache, void* value_cache,
    const int32_t* block_tables, const int32_t* context_lens, int num_seqs, int num_heads,
    int num_kv_heads, int head_size, int block_size, int max_blocks_per_seq, int max_context,
    float scale, int kv_head_map, int dtype, void* workspace, size_t workspace_bytes,
    lmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LMRS_DECODE_H */
