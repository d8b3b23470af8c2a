// decode_layer_capi.cuh — the C-ABI of include/lmrs_layer.h (included at the end
// of lmrs_capi.cu, one translation unit with the other entry points).
#pragma once
#include <algorithm>
#include <tuple>
#include <vector>

#include "decode_layer.cuh"
#include "lmrs_layer.h"

namespace {

constexpr int kDlAreaMax = 96 * 1024;

// Shapes -> launch geometry and workspace layout for a grid of G CTAs.
struct DlPlan {
  int G, M, H, hq, hkv, inter, chunk, nchunk, ring, area, smem;
  int N[4], K[4];
  size_t off_ss, off_max, off_sched, off_xrow, off_qkv, off_gu, off_obuf, off_atto, off_attml,
      off_trace, total;
  int sched_ints;
};

size_t dl_align(size_t v) { return (v + 255) & ~size_t(255); }

int dl_plan(const lmrs_fp8_layer_shape_t* s, int G, DlPlan* p) {
  if (!s) return LMRS_ERR_NULL;
  const int M = s->num_seqs, H = s->hidden, hq = s->num_heads, hkv = s->num_kv_heads;
  const int I = s->intermediate;
  if (M < 1 || M > lmrs::kDlMaxTok || s->head_size != lmrs::kDlD || hkv < 1 || hq < hkv ||
      hq % hkv || hq / hkv > lmrs::kDlMaxGroup || H < 128 || H % 128 || I < 128 || I % 128 ||
      s->block_size < 1 || s->max_blocks_per_seq < 1 || s->max_context < 1 ||
      static_cast<long long>(s->block_size) * s->max_blocks_per_seq > INT32_MAX ||
      !(s->eps >= 0.f) || G < 1 || G > lmrs::kDlMaxGrid)
    return LMRS_ERR_SHAPE;
  p->G = G;
  p->M = M;
  p->H = H;
  p->hq = hq;
  p->hkv = hkv;
  p->inter = I;
  const int d = lmrs::kDlD;
  p->N[0] = (hq + 2 * hkv) * d;
  p->K[0] = H;
  p->N[1] = H;
  p->K[1] = hq * d;
  p->N[2] = 2 * I;
  p->K[2] = H;
  p->N[3] = H;
  p->K[3] = I;
  const int kmax = std::max(std::max(H, hq * d), I);
  if (static_cast<long long>(M) * (kmax + 16) > kDlAreaMax) return LMRS_ERR_SHAPE;
  // attention units: (token, KV head, chunk) about one per CTA, 16..64 positions each
  const long long work = static_cast<long long>(M) * hkv * s->max_context;
  int chunk = static_cast<int>((work + G - 1) / G);
  chunk = (chunk + 15) / 16 * 16;
  p->chunk = std::min(std::max(chunk, 16), lmrs::kDlMaxChunk);
  p->nchunk = (s->max_context + p->chunk - 1) / p->chunk;
  p->area = std::max(M * (kmax + 16), lmrs::kDlAttnBytes);
  p->area = (p->area + 127) / 128 * 128;
  const int fixed = lmrs::dl_smem_bytes(0, p->area);
  p->ring = std::min((227 * 1024 - fixed) / (lmrs::kDlSlot + 16), 12);
  if (p->ring < 2 || p->ring * lmrs::kDlSlot < 64 * 1024) return LMRS_ERR_SHAPE;
  p->smem = lmrs::dl_smem_bytes(p->ring, p->area);
  int units = 0;
  for (int q = 0; q < 4; ++q) units += p->N[q] / lmrs::kDlRows;
  p->sched_ints = 4 * (G + 1) + units;
  const int Gq = hq / hkv;
  size_t off = 256;  // barrier counter
  p->off_ss = off;
  off = dl_align(off + size_t(G) * lmrs::kDlMaxTok * 4);
  p->off_max = off;
  off = dl_align(off + size_t(G) * lmrs::kDlMaxTok * 4);
  p->off_sched = off;
  off = dl_align(off + size_t(p->sched_ints) * 4);
  p->off_xrow = off;
  off = dl_align(off + size_t(M) * kmax * 2);
  p->off_qkv = off;
  off = dl_align(off + size_t(M) * p->N[0] * 2);
  p->off_gu = off;
  off = dl_align(off + size_t(M) * p->N[2] * 2);
  p->off_obuf = off;
  off = dl_align(off + size_t(M) * H * 2);
  p->off_atto = off;
  const size_t parts = size_t(M) * hkv * p->nchunk * Gq;
  off = dl_align(off + parts * d * 4);
  p->off_attml = off;
  off = dl_align(off + parts * 2 * 4);
  p->off_trace = off;  // phase timestamps when the "decode_layer_trace" knob is on
  off = dl_align(off + size_t(G) * lmrs::kDlTraceSlots * 8);
  p->total = off;
  return LMRS_OK;
}

// Units of 16 weight rows, phase by phase: each to the CTA with the fewest
// units of this phase, then the fewest weight bytes so far, then the lowest
// index, so that every phase is spread over all CTAs (its latency is the
// busiest CTA's) and the extra units of one phase land on CTAs that had fewer
// bytes before.  Layout: [4][G + 1] offsets into the unit list that follows
// (each CTA's units ascending).
std::vector<int> dl_schedule(const DlPlan& p) {
  const int G = p.G;
  std::vector<int> out(p.sched_ints, 0);
  std::vector<long long> load(G, 0);
  int next = 4 * (G + 1);
  for (int q = 0; q < 4; ++q) {
    const int nu = p.N[q] / lmrs::kDlRows;
    const long long bytes = static_cast<long long>(lmrs::kDlRows) * p.K[q];
    std::vector<int> owner(nu);
    using Item = std::tuple<int, long long, int>;  // (units this phase, bytes so far, CTA)
    std::vector<Item> heap;
    heap.reserve(G);
    for (int c = 0; c < G; ++c) heap.emplace_back(0, load[c], c);
    auto cmp = [](const Item& a, const Item& b) { return a > b; };  // min-heap
    std::make_heap(heap.begin(), heap.end(), cmp);
    for (int u = 0; u < nu; ++u) {
      std::pop_heap(heap.begin(), heap.end(), cmp);
      Item& it = heap.back();
      owner[u] = std::get<2>(it);
      std::get<0>(it) += 1;
      std::get<1>(it) += bytes;
      std::push_heap(heap.begin(), heap.end(), cmp);
    }
    for (const Item& it : heap) load[std::get<2>(it)] = std::get<1>(it);
    std::vector<int> count(G, 0);
    for (int u = 0; u < nu; ++u) ++count[owner[u]];
    int* offs = out.data() + q * (G + 1);
    offs[0] = next;
    for (int c = 0; c < G; ++c) offs[c + 1] = offs[c] + count[c];
    std::vector<int> fill(offs, offs + G);
    for (int u = 0; u < nu; ++u) out[fill[owner[u]]++] = u;
    next = offs[G];
  }
  // offsets relative to the start of the unit list
  for (int q = 0; q < 4; ++q)
    for (int c = 0; c <= G; ++c) out[q * (G + 1) + c] -= 4 * (G + 1);
  return out;
}

int dl_grid(int dev) { return std::min(sm_count(dev), lmrs::kDlMaxGrid); }

// An e4m3 weight [N][K] as the 3-D tensor [N][K / 128][128] bytes, box [16][8][128]
// (one ring slot: 16 rows x 1024 bytes of K; K / 128 not a multiple of 8 leaves
// the last box's tail zero-filled).
int dl_weight_map(CUtensorMap* m, const uint8_t* w, int N, int K) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMRS_ERR_CUDA;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(K / 128), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(K)};
  cuuint32_t box[3] = {128, lmrs::kDlSeg / 128, lmrs::kDlRows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(w), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return LMRS_ERR_CUDA;
  }
  return LMRS_OK;
}

}  // namespace

extern "C" {

LMRS_API size_t lmrs_fp8_decode_layer_workspace_bytes(const lmrs_fp8_layer_shape_t* shape) {
  int dev = 0;
  if (check_device(&dev)) return 0;
  DlPlan p;
  if (dl_plan(shape, dl_grid(dev), &p)) return 0;
  return p.total;
}

LMRS_API int lmrs_fp8_decode_layer_prepare(const lmrs_fp8_layer_shape_t* shape, void* workspace,
                                           size_t workspace_bytes, lmrs_stream_t stream) {
  int dev = 0, rc;
  DlPlan p;
  if ((rc = dl_plan(shape, 1, &p))) return rc;
  if (!workspace) return LMRS_ERR_WORKSPACE;
  if ((rc = check_device(&dev))) return rc;
  if ((rc = dl_plan(shape, dl_grid(dev), &p))) return rc;
  if (workspace_bytes < p.total) return LMRS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return LMRS_ERR_ALIGN;
  const std::vector<int> sched = dl_schedule(p);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(ws, 0, p.off_sched, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(ws + p.off_sched, sched.data(), sched.size() * sizeof(int),
                        cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // `sched` is pageable and local
  return e == cudaSuccess ? LMRS_OK : record(e);
}

LMRS_API int lmrs_fp8_decode_layer(const lmrs_fp8_layer_t* layer,
                                   const lmrs_fp8_layer_shape_t* shape, void* residual,
                                   const void* delta_in_or_null, void* delta_out, int flags,
                                   const int32_t* block_tables, const int32_t* context_lens,
                                   const void* cos, const void* sin, int rank, int world,
                                   void* const* buffers, size_t max_elems, void* workspace,
                                   size_t workspace_bytes, lmrs_stream_t stream) {
  int dev = 0, rc;
  if (!layer) return LMRS_ERR_NULL;
  DlPlan p;
  if ((rc = dl_plan(shape, 1, &p))) return rc;  // the shape rules (no device needed)
  if (world < 1 || world > lmrs::kArMaxRanks || rank < 0 || rank >= world ||
      (flags & ~(LMRS_LAYER_RECV_DELTA | LMRS_LAYER_PUSH_DELTA)) ||
      (world == 1 && flags != 0))
    return LMRS_ERR_SHAPE;
  const void* ptrs[] = {layer->qkv_weight, layer->qkv_scale, layer->o_weight, layer->o_scale,
                        layer->gate_up_weight, layer->gate_up_scale, layer->down_weight,
                        layer->down_scale, layer->input_norm, layer->post_norm,
                        layer->key_cache, layer->value_cache, residual, delta_out,
                        block_tables, context_lens, cos, sin, workspace};
  for (const void* q : ptrs)
    if (!q) return LMRS_ERR_NULL;
  const void* al[] = {layer->qkv_weight, layer->o_weight, layer->gate_up_weight,
                      layer->down_weight, layer->input_norm, layer->post_norm,
                      layer->key_cache, layer->value_cache, residual, delta_out, cos, sin};
  for (const void* q : al)
    if (!aligned16(q)) return LMRS_ERR_ALIGN;
  if (delta_in_or_null && !aligned16(delta_in_or_null)) return LMRS_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return LMRS_ERR_ALIGN;
  if (world > 1) {
    if (!buffers) return LMRS_ERR_NULL;
    for (int r = 0; r < world; ++r)
      if (!buffers[r]) return LMRS_ERR_NULL;
    if (max_elems / 2 > static_cast<size_t>(INT32_MAX) ||
        static_cast<size_t>(p.M) * static_cast<size_t>(p.H) > max_elems)
      return LMRS_ERR_SHAPE;
  }
  if ((rc = check_device(&dev))) return rc;
  if ((rc = dl_plan(shape, dl_grid(dev), &p))) return rc;
  if (workspace_bytes < p.total) return LMRS_ERR_WORKSPACE;

  lmrs::DlArgs a = {};
  a.w[0] = layer->qkv_weight;
  a.w[1] = layer->o_weight;
  a.w[2] = layer->gate_up_weight;
  a.w[3] = layer->down_weight;
  a.sw[0] = layer->qkv_scale;
  a.sw[1] = layer->o_scale;
  a.sw[2] = layer->gate_up_scale;
  a.sw[3] = layer->down_scale;
  for (int q = 0; q < 4; ++q) {
    a.N[q] = p.N[q];
    a.K[q] = p.K[q];
    if ((rc = dl_weight_map(&a.tm[q], a.w[q], p.N[q], p.K[q]))) return rc;
  }
  a.in_norm = static_cast<const __nv_bfloat16*>(layer->input_norm);
  a.post_norm = static_cast<const __nv_bfloat16*>(layer->post_norm);
  a.kc = static_cast<__nv_bfloat16*>(layer->key_cache);
  a.vc = static_cast<__nv_bfloat16*>(layer->value_cache);
  a.tables = block_tables;
  a.ctx_lens = context_lens;
  a.cosv = static_cast<const __nv_bfloat16*>(cos);
  a.sinv = static_cast<const __nv_bfloat16*>(sin);
  a.resid = static_cast<__nv_bfloat16*>(residual);
  a.delta_in = static_cast<const __nv_bfloat16*>(delta_in_or_null);
  a.delta_out = static_cast<__nv_bfloat16*>(delta_out);
  a.M = p.M;
  a.H = p.H;
  a.hq = p.hq;
  a.hkv = p.hkv;
  a.inter = p.inter;
  a.block_size = shape->block_size;
  a.max_blocks = shape->max_blocks_per_seq;
  a.chunk = p.chunk;
  a.nchunk = p.nchunk;
  a.ring = p.ring;
  a.area = p.area;
  a.eps = shape->eps;
  a.scale_log2 = shape->scale * 1.4426950408889634f;
  a.rank = rank;
  a.world = world;
  a.recv_delta = (flags & LMRS_LAYER_RECV_DELTA) ? 1 : 0;
  a.push_delta = (flags & LMRS_LAYER_PUSH_DELTA) ? 1 : 0;
  a.cap = world > 1 ? static_cast<int>(ar_cap(max_elems)) : 0;
  for (int r = 0; r < world && world > 1; ++r)
    a.peers.buf[r] = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(buffers[r]) + kArHeader);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.bar = reinterpret_cast<unsigned long long*>(ws);
  a.st_ss = reinterpret_cast<float*>(ws + p.off_ss);
  a.st_max = reinterpret_cast<float*>(ws + p.off_max);
  a.sched = reinterpret_cast<const int*>(ws + p.off_sched);
  a.xrow = reinterpret_cast<__nv_bfloat16*>(ws + p.off_xrow);
  a.qkv = reinterpret_cast<__nv_bfloat16*>(ws + p.off_qkv);
  a.gu = reinterpret_cast<__nv_bfloat16*>(ws + p.off_gu);
  a.obuf = reinterpret_cast<__nv_bfloat16*>(ws + p.off_obuf);
  a.att_o = reinterpret_cast<float*>(ws + p.off_atto);
  a.att_ml = reinterpret_cast<float*>(ws + p.off_attml);
  a.trace = g_tune.decode_layer_trace ? reinterpret_cast<unsigned long long*>(ws + p.off_trace)
                                      : nullptr;

  if ((rc = ensure_smem_of<lmrs::fp8_decode_layer_kernel>(p.smem, dev))) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.G, 1, 1);
  cfg.blockDim = dim3(lmrs::kDlThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lmrs::fp8_decode_layer_kernel, a);
  if (e != cudaSuccess) return record(e);
  return after_launch();
}

}  // extern "C"
