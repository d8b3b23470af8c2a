// decode_capi.cuh — the C-ABI of include/lmrs_decode.h.  Included at the end of
// lmrs_capi.cu (one translation unit: shares its launch helpers and checks).
#pragma once
#include "decode_ops.cuh"
#include "lmrs_decode.h"

namespace {

bool act_dtype(int dt) { return dt == LMRS_DTYPE_BF16 || dt == LMRS_DTYPE_F16; }

// A whole row in one CTA's registers: the fewest vectors per thread (1, 2 or 4
// of 8 columns) that fit 1024 threads, and the threads that covers.
constexpr int kRowMaxCols = lmrs::kRowMaxThreads * lmrs::kRowMaxVecs * 8;

void row_shape(int cols, int* vpt, int* threads) {
  const int vecs = cols / 8;
  int v = 1;
  while (v < lmrs::kRowMaxVecs && vecs > lmrs::kRowMaxThreads * v) v *= 2;
  int t = (vecs + v - 1) / v;
  t = (t + 31) / 32 * 32;
  *vpt = v;
  *threads = clampi(t, lmrs::kNormThreads, lmrs::kRowMaxThreads);
}

template <typename T, bool FP8>
int rmsnorm_launch(void* out, uint8_t* q, float* s, void* resid, const void* delta, const void* w,
                   int rows, int H, float eps, cudaStream_t st) {
  int vpt, threads;
  row_shape(H, &vpt, &threads);
  auto go = [&](auto kern) {
    return launch_ex_grid(kern, dim3(rows, 1, 1), threads, st, static_cast<T*>(out), q, s,
                          static_cast<T*>(resid), static_cast<const T*>(delta),
                          static_cast<const T*>(w), H, eps);
  };
  int rc = vpt == 1   ? go(lmrs::rmsnorm_kernel<T, FP8, 1>)
           : vpt == 2 ? go(lmrs::rmsnorm_kernel<T, FP8, 2>)
                      : go(lmrs::rmsnorm_kernel<T, FP8, 4>);
  return rc ? rc : after_launch();
}

template <typename T, bool FP8>
int silu_launch(void* out, uint8_t* q, float* s, const void* gu, int rows, int inter,
                cudaStream_t st) {
  int rc;
  if (!FP8) {  // no row reduction: (row, chunk of 256 x 8 columns) CTAs
    const int chunks = (inter + lmrs::kNormThreads * 8 - 1) / (lmrs::kNormThreads * 8);
    rc = launch_ex_grid(lmrs::silu_mul_kernel<T, FP8, 1>, dim3(rows, chunks, 1),
                        lmrs::kNormThreads, st, static_cast<T*>(out), q, s,
                        static_cast<const T*>(gu), inter);
  } else if (inter > lmrs::kSiluClusterThreads * lmrs::kSiluClusterVecs * 8) {
    // long rows: a cluster of CTAs per row, absmax exchanged through DSMEM
    const int per = lmrs::kSiluClusterThreads * lmrs::kSiluClusterVecs * 8;
    const int C = (inter + per - 1) / per;
    rc = launch_ex_cluster3(lmrs::silu_mul_fp8_cluster_kernel<T>, dim3(rows, C, 1), dim3(1, C, 1),
                            lmrs::kSiluClusterThreads, st, q, s, static_cast<const T*>(gu), inter);
  } else {
    int vpt, threads;
    row_shape(inter, &vpt, &threads);
    auto go = [&](auto kern) {
      return launch_ex_grid(kern, dim3(rows, 1, 1), threads, st, static_cast<T*>(out), q, s,
                            static_cast<const T*>(gu), inter);
    };
    rc = vpt == 1   ? go(lmrs::silu_mul_kernel<T, FP8, 1>)
         : vpt == 2 ? go(lmrs::silu_mul_kernel<T, FP8, 2>)
                    : go(lmrs::silu_mul_kernel<T, FP8, 4>);
  }
  return rc ? rc : after_launch();
}

// context split of the decode attention: as many splits as keep the grid within
// one wave of ~2 CTAs per SM (rounded down: 128 (sequence, KV head) pairs at
// batch 16 run 2 splits in 32.6 us against 44.8 us for 3, which spill into a
// second wave), whole 64-position tiles.  Up to kAttnMaxCluster splits merge in
// one cluster's shared memory; more (small batches) come in whole clusters
// (splits a multiple of kAttnMaxCluster, trailing splits possibly empty) whose
// merged partials meet in the workspace.
struct AttnSplit {
  int splits, span;
  int clusters;   // clusters per (sequence, KV head); > 1 needs the workspace
};

AttnSplit attn_split(int seqs, int hkv, int max_ctx, int sms) {
  const int tiles = max_ctx > 0 ? (max_ctx + lmrs::kAttnTile - 1) / lmrs::kAttnTile : 1;  // 64-pos units
  const int work = seqs * hkv > 0 ? seqs * hkv : 1;
  int s = clampi((g_tune.attn_ctas_per_sm * sms) / work, 1, tiles);
  // several clusters only for long contexts: B=1, 8 KV heads, 2048 positions
  // took 9.1 us on one cluster of 8 splits against 11.4 us on 4 clusters; at
  // 4096 positions 13.8 against 13.0, and 13.6 against 9.4 with one KV head
  const bool multi = g_tune.attn_global_merge && max_ctx > g_tune.attn_multi_min_ctx;
  const int cap = multi ? lmrs::kAttnMaxSplits : lmrs::kAttnMaxCluster;
  if (s > cap) s = cap;
  if (s > lmrs::kAttnMaxCluster) s -= s % lmrs::kAttnMaxCluster;   // whole clusters
  const int per = (tiles + s - 1) / s;
  AttnSplit r;
  r.span = per * lmrs::kAttnTile;
  r.splits = (tiles + per - 1) / per;
  if (r.splits > lmrs::kAttnMaxCluster)
    r.splits = static_cast<int>(round_up(size_t(r.splits), lmrs::kAttnMaxCluster));
  r.clusters = r.splits > lmrs::kAttnMaxCluster ? r.splits / lmrs::kAttnMaxCluster : 1;
  return r;
}

// Workspace of the second merge level: the cluster partials [seqs * hkv]
// [clusters][16 rows][132] fp32, then one arrival counter per (sequence, KV head).
size_t attn_ws_part_bytes(int seqs, int hkv, const AttnSplit& sp) {
  return round_up(size_t(seqs) * hkv * sp.clusters * 16 * lmrs::kAttnPartStride * 4, 256);
}

size_t attn_ws_bytes(int seqs, int hkv, const AttnSplit& sp) {
  if (sp.clusters == 1) return 0;
  return attn_ws_part_bytes(seqs, hkv, sp) + round_up(size_t(seqs) * hkv * 4, 256);
}

std::atomic<int> g_smem_attn[2][2][3][kMaxDevices];  // [dtype][rope][stages - 2]

// ROPE: q is the merged qkv row and cosv / sinv the RoPE tables (the fused
// RoPE + KV write); otherwise q holds the query rows and cosv / sinv are null.
template <typename T, int NS, bool ROPE>
int attn_launch(void* out, const void* q, const void* kc, const void* vc,
                const int32_t* tables, const int32_t* lens, int seqs, int heads, int hkv,
                int bs, int maxb, const AttnSplit& sp, float scale, int map, void* ws,
                cudaStream_t st, int dev, std::atomic<int>* done, uint8_t* qout, float* qscale,
                const void* cosv, const void* sinv) {
  const int splits = sp.splits, span = sp.span;
  float* ws_part = nullptr;
  uint32_t* ws_count = nullptr;
  if (sp.clusters > 1) {
    ws_part = static_cast<float*>(ws);
    ws_count = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + attn_ws_part_bytes(seqs, hkv, sp));
  }
  int rc;
  if ((rc = ensure_smem(lmrs::decode_attn_kernel<T, NS, ROPE>, lmrs::attn_smem_bytes(NS), done,
                        dev)))
    return rc;
  const float scale_log2 = scale * 1.4426950408889634f;
  // grid (seqs * hkv, splits): launch_ex is 1-D, so pack the split into y here
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(seqs * hkv, splits, 1);
  c.blockDim = dim3(lmrs::kAttnThreads, 1, 1);
  c.dynamicSmemBytes = lmrs::attn_smem_bytes(NS);
  c.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (splits > 1) {   // consecutive splits of one (sequence, KV head) merge inside their cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = splits < lmrs::kAttnMaxCluster ? splits : lmrs::kAttnMaxCluster;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (g_tune.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  c.attrs = attr;
  c.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(
      &c, lmrs::decode_attn_kernel<T, NS, ROPE>, static_cast<T*>(out), static_cast<const T*>(q),
      static_cast<const T*>(kc), static_cast<const T*>(vc), tables, lens, heads, hkv, bs, maxb,
      span, scale_log2, map, ws_part, ws_count, qout, qscale, static_cast<const T*>(cosv),
      static_cast<const T*>(sinv), const_cast<T*>(static_cast<const T*>(kc)),
      const_cast<T*>(static_cast<const T*>(vc)));
  if (e != cudaSuccess) return record(e);
  return after_launch();
}

}  // namespace

extern "C" {

LMRS_API int lmrs_rmsnorm(void* out, void* residual, const void* delta_or_null, const void* weight,
                          int rows, int H, float eps, int dtype, lmrs_stream_t stream) {
  if (!act_dtype(dtype)) return LMRS_ERR_DTYPE;
  if (rows < 0 || H <= 0 || H % 8 || H > kRowMaxCols) return LMRS_ERR_SHAPE;
  if (rows == 0) return LMRS_OK;
  if (!out || !residual || !weight) return LMRS_ERR_NULL;
  if (!aligned16(out) || !aligned16(residual) || !aligned16(weight) ||
      (delta_or_null && !aligned16(delta_or_null)))
    return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? rmsnorm_launch<__nv_bfloat16, false>(out, nullptr, nullptr, residual, delta_or_null,
                                                    weight, rows, H, eps, st)
             : rmsnorm_launch<__half, false>(out, nullptr, nullptr, residual, delta_or_null,
                                             weight, rows, H, eps, st);
}

LMRS_API int lmrs_rmsnorm_fp8(uint8_t* q_out, float* scale_out, void* residual,
                              const void* delta_or_null, const void* weight, int rows, int H,
                              float eps, int dtype, lmrs_stream_t stream) {
  if (!act_dtype(dtype)) return LMRS_ERR_DTYPE;
  if (rows < 0 || H <= 0 || H % 8 || H > kRowMaxCols) return LMRS_ERR_SHAPE;
  if (rows == 0) return LMRS_OK;
  if (!q_out || !scale_out || !residual || !weight) return LMRS_ERR_NULL;
  if (!aligned16(q_out) || !aligned16(residual) || !aligned16(weight) ||
      (delta_or_null && !aligned16(delta_or_null)))
    return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? rmsnorm_launch<__nv_bfloat16, true>(nullptr, q_out, scale_out, residual,
                                                   delta_or_null, weight, rows, H, eps, st)
             : rmsnorm_launch<__half, true>(nullptr, q_out, scale_out, residual, delta_or_null,
                                            weight, rows, H, eps, st);
}

LMRS_API int lmrs_silu_mul(void* out, const void* gate_up, int rows, int inter, int dtype,
                           lmrs_stream_t stream) {
  if (!act_dtype(dtype)) return LMRS_ERR_DTYPE;
  if (rows < 0 || inter <= 0 || inter % 8) return LMRS_ERR_SHAPE;
  if (rows == 0) return LMRS_OK;
  if (!out || !gate_up) return LMRS_ERR_NULL;
  if (!aligned16(out) || !aligned16(gate_up)) return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? silu_launch<__nv_bfloat16, false>(out, nullptr, nullptr, gate_up, rows, inter, st)
             : silu_launch<__half, false>(out, nullptr, nullptr, gate_up, rows, inter, st);
}

LMRS_API int lmrs_silu_mul_fp8(uint8_t* q_out, float* scale_out, const void* gate_up, int rows,
                               int inter, int dtype, lmrs_stream_t stream) {
  if (!act_dtype(dtype)) return LMRS_ERR_DTYPE;
  if (rows < 0 || inter <= 0 || inter % 8 ||
      inter > lmrs::kSiluMaxCluster * lmrs::kSiluClusterThreads * lmrs::kSiluClusterVecs * 8)
    return LMRS_ERR_SHAPE;
  if (rows == 0) return LMRS_OK;
  if (!q_out || !scale_out || !gate_up) return LMRS_ERR_NULL;
  if (!aligned16(q_out) || !aligned16(gate_up)) return LMRS_ERR_ALIGN;
  int rc = check_device(nullptr);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == LMRS_DTYPE_BF16
             ? silu_launch<__nv_bfloat16, true>(nullptr, q_out, scale_out, gate_up, rows, inter, st)
             : silu_launch<__half, true>(nullptr, q_out, scale_out, gate_up, rows, inter, st);
}

LMRS_API int lmrs_rope_kv_write(void* q_out, void* key_cache, void* value_cache, const void* qkv,
                                const void* cos, const void* sin, const int32_t* block_tables,
                                const int32_t* positions, int num_seqs, int num_heads,
                                int num_kv_heads, int head_size, int block_size,
                                int max_blocks_per_seq, int dtype, lmrs_stream_t stream) {
  if (!act_dtype(dtype)) return LMRS_ERR_DTYPE;
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_size <= 0 || head_size % 2 ||
      block_size <= 0 || max_blocks_per_seq <= 0)
    return LMRS_ERR_SHAPE;
  if (num_seqs == 0) return LMRS_OK;
  if (!q_out || !key_cache || !value_cache || !qkv || !cos || !sin || !block_tables || !positions)
    return LMRS_ERR_NULL;
  int rc = check_device(nullptr);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = head_size % 16 == 0 && aligned16(q_out) && aligned16(key_cache) &&
                   aligned16(value_cache) && aligned16(qkv) && aligned16(cos) && aligned16(sin);
  const int items = (num_heads + num_kv_heads) * (head_size / 16) + num_kv_heads * (head_size / 8);
  const dim3 vgrid(num_seqs, (items + 127) / 128, 1);
  auto go = [&](auto tag) {
    using T = decltype(tag);
    if (vec)
      return launch_ex_grid(lmrs::rope_kv_vec_kernel<T>, vgrid, 128, st, static_cast<T*>(q_out),
                            static_cast<T*>(key_cache), static_cast<T*>(value_cache),
                            static_cast<const T*>(qkv), static_cast<const T*>(cos),
                            static_cast<const T*>(sin), block_tables, positions, num_heads,
                            num_kv_heads, head_size, block_size, max_blocks_per_seq);
    return launch_ex(lmrs::rope_kv_kernel<T>, num_seqs, 0, 256, 0, st, static_cast<T*>(q_out),
                     static_cast<T*>(key_cache), static_cast<T*>(value_cache),
                     static_cast<const T*>(qkv), static_cast<const T*>(cos),
                     static_cast<const T*>(sin), block_tables, positions, num_heads, num_kv_heads,
                     head_size, block_size, max_blocks_per_seq);
  };
  rc = dtype == LMRS_DTYPE_BF16 ? go(__nv_bfloat16()) : go(__half());
  return rc ? rc : after_launch();
}

LMRS_API size_t lmrs_paged_attention_workspace_bytes(int num_seqs, int num_heads,
                                                     int num_kv_heads, int max_context) {
  (void)num_heads;
  if (num_seqs <= 0 || num_kv_heads <= 0 || max_context < 0) return 0;
  return attn_ws_bytes(num_seqs, num_kv_heads,
                       attn_split(num_seqs, num_kv_heads, max_context, sm_count_cached()));
}

}  // extern "C"

namespace {

int paged_attention_impl(void* out, const void* query, const void* key_cache,
                         const void* value_cache, const int32_t* block_tables,
                         const int32_t* context_lens, int num_seqs, int num_heads,
                         int num_kv_heads, int head_size, int block_size, int max_blocks_per_seq,
                         int max_context, float scale, int kv_head_map, int dtype,
                         void* workspace, size_t workspace_bytes, lmrs_stream_t stream,
                         uint8_t* qout, float* qscale, const void* cosv = nullptr,
                         const void* sinv = nullptr) {
  if (!act_dtype(dtype)) return LMRS_ERR_DTYPE;
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads ||
      num_heads / num_kv_heads > 16 || head_size != lmrs::kAttnD || block_size <= 0 ||
      max_blocks_per_seq <= 0 || max_context < 0 || (kv_head_map != 0 && kv_head_map != 1))
    return LMRS_ERR_SHAPE;
  if (num_seqs == 0) return LMRS_OK;
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens)
    return LMRS_ERR_NULL;
  if (!aligned16(out) || !aligned16(query) || !aligned16(key_cache) || !aligned16(value_cache))
    return LMRS_ERR_ALIGN;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc) return rc;
  const AttnSplit sp = attn_split(num_seqs, num_kv_heads, max_context, sm_count(dev));
  if (sp.clusters > 1) {
    if (!workspace || workspace_bytes < attn_ws_bytes(num_seqs, num_kv_heads, sp))
      return LMRS_ERR_WORKSPACE;
    if (!aligned16(workspace)) return LMRS_ERR_ALIGN;
  }
  const int ns = clampi(g_tune.attn_stages, 2, 4);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define LMRS_ATTN(T, I, NS)                                                                      \
  return cosv != nullptr                                                                         \
             ? attn_launch<T, NS, true>(out, query, key_cache, value_cache, block_tables,       \
                                        context_lens, num_seqs, num_heads, num_kv_heads,        \
                                        block_size, max_blocks_per_seq, sp, scale, kv_head_map, \
                                        workspace, st, dev, g_smem_attn[I][1][NS - 2], qout,    \
                                        qscale, cosv, sinv)                                     \
             : attn_launch<T, NS, false>(out, query, key_cache, value_cache, block_tables,      \
                                         context_lens, num_seqs, num_heads, num_kv_heads,       \
                                         block_size, max_blocks_per_seq, sp, scale,             \
                                         kv_head_map, workspace, st, dev,                       \
                                         g_smem_attn[I][0][NS - 2], qout, qscale, nullptr,      \
                                         nullptr)
  if (dtype == LMRS_DTYPE_BF16) {
    if (ns == 2) LMRS_ATTN(__nv_bfloat16, 0, 2);
    if (ns == 3) LMRS_ATTN(__nv_bfloat16, 0, 3);
    LMRS_ATTN(__nv_bfloat16, 0, 4);
  }
  if (ns == 2) LMRS_ATTN(__half, 1, 2);
  if (ns == 3) LMRS_ATTN(__half, 1, 3);
  LMRS_ATTN(__half, 1, 4);
#undef LMRS_ATTN
}

}  // namespace

extern "C" {

LMRS_API int lmrs_paged_attention_decode(void* out, const void* query, const void* key_cache,
                                         const void* value_cache, const int32_t* block_tables,
                                         const int32_t* context_lens, int num_seqs, int num_heads,
                                         int num_kv_heads, int head_size, int block_size,
                                         int max_blocks_per_seq, int max_context, float scale,
                                         int kv_head_map, int dtype, void* workspace,
                                         size_t workspace_bytes, lmrs_stream_t stream) {
  return paged_attention_impl(out, query, key_cache, value_cache, block_tables, context_lens,
                              num_seqs, num_heads, num_kv_heads, head_size, block_size,
                              max_blocks_per_seq, max_context, scale, kv_head_map, dtype,
                              workspace, workspace_bytes, stream, nullptr, nullptr);
}

// One KV head (tensor-parallel ranks of GQA models with as many ranks as KV
// heads): the attention's final merge holds whole token rows and emits their
// e4m3 bytes and scales itself; otherwise the attention, then the row quant.
LMRS_API int lmrs_paged_attention_decode_fp8(uint8_t* q_out, float* scale_out, void* out,
                                             const void* query, const void* key_cache,
                                             const void* value_cache, const int32_t* block_tables,
                                             const int32_t* context_lens, int num_seqs,
                                             int num_heads, int num_kv_heads, int head_size,
                                             int block_size, int max_blocks_per_seq,
                                             int max_context, float scale, int kv_head_map,
                                             int dtype, void* workspace, size_t workspace_bytes,
                                             lmrs_stream_t stream) {
  if (num_seqs > 0 && (!q_out || !scale_out)) return LMRS_ERR_NULL;
  if (q_out && !aligned16(q_out)) return LMRS_ERR_ALIGN;
  if (num_kv_heads == 1)
    return paged_attention_impl(out, query, key_cache, value_cache, block_tables, context_lens,
                                num_seqs, num_heads, num_kv_heads, head_size, block_size,
                                max_blocks_per_seq, max_context, scale, kv_head_map, dtype,
                                workspace, workspace_bytes, stream, q_out, scale_out);
  int rc = paged_attention_impl(out, query, key_cache, value_cache, block_tables, context_lens,
                                num_seqs, num_heads, num_kv_heads, head_size, block_size,
                                max_blocks_per_seq, max_context, scale, kv_head_map, dtype,
                                workspace, workspace_bytes, stream, nullptr, nullptr);
  if (rc || num_seqs == 0) return rc;
  return lmrs_fp8_quant_rows(q_out, scale_out, out, num_seqs, num_heads * head_size, dtype,
                             stream);
}

// RoPE + KV-cache write of the new token (position context_lens - 1) fused into
// the attention: lmrs_rope_kv_write (positions = context_lens - 1) then
// lmrs_paged_attention_decode[_fp8] in one launch (two with an FP8 output and
// more than one KV head).
LMRS_API int lmrs_rope_paged_attention_decode(
    void* out, uint8_t* q_out_or_null, float* scale_out_or_null, const void* qkv,
    const void* cos, const void* sin, void* key_cache, void* value_cache,
    const int32_t* block_tables, const int32_t* context_lens, int num_seqs, int num_heads,
    int num_kv_heads, int head_size, int block_size, int max_blocks_per_seq, int max_context,
    float scale, int kv_head_map, int dtype, void* workspace, size_t workspace_bytes,
    lmrs_stream_t stream) {
  if (num_seqs > 0 && (!cos || !sin)) return LMRS_ERR_NULL;
  if ((cos && !aligned16(cos)) || (sin && !aligned16(sin))) return LMRS_ERR_ALIGN;
  const bool fp8 = q_out_or_null != nullptr;
  if (fp8 && num_seqs > 0 && !scale_out_or_null) return LMRS_ERR_NULL;
  if (fp8 && !aligned16(q_out_or_null)) return LMRS_ERR_ALIGN;
  const bool fused_q = fp8 && num_kv_heads == 1;
  int rc = paged_attention_impl(out, qkv, key_cache, value_cache, block_tables, context_lens,
                                num_seqs, num_heads, num_kv_heads, head_size, block_size,
                                max_blocks_per_seq, max_context, scale, kv_head_map, dtype,
                                workspace, workspace_bytes, stream,
                                fused_q ? q_out_or_null : nullptr,
                                fused_q ? scale_out_or_null : nullptr, cos, sin);
  if (rc || !fp8 || fused_q || num_seqs == 0) return rc;
  return lmrs_fp8_quant_rows(q_out_or_null, scale_out_or_null, out, num_seqs,
                             num_heads * head_size, dtype, stream);
}

}  // extern "C"
