// awq_pack.cuh — AWQ int4 unpack and bit-exact fp16 dequant kernels.
//
// Both are pure streaming kernels (one packed int32 word per thread, 4 B in,
// 8 B or 16 B out), bounded by HBM bandwidth; consecutive threads touch
// consecutive words, so every load and store is fully coalesced.
#pragma once
#include "lmrs_ptx.cuh"

namespace lmrs {

// q_out[r, 8j + ORDER[i]] = nibble i of packed[r, j].
__global__ void __launch_bounds__(256) awq_unpack_kernel(int8_t* __restrict__ q_out,
                                                         const uint32_t* __restrict__ packed,
                                                         int64_t total_words) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total_words) return;
  const uint32_t w = __ldg(packed + idx);
  // column c lives in nibble INV[c], INV = {0,4,1,5,2,6,3,7}
  uint32_t lo = ((w >> 0) & 0xFu) | (((w >> 16) & 0xFu) << 8) | (((w >> 4) & 0xFu) << 16) |
                (((w >> 20) & 0xFu) << 24);
  uint32_t hi = ((w >> 8) & 0xFu) | (((w >> 24) & 0xFu) << 8) | (((w >> 12) & 0xFu) << 16) |
                (((w >> 28) & 0xFu) << 24);
  reinterpret_cast<uint2*>(q_out)[idx] = make_uint2(lo, hi);
}

// w_out[k, n] = T_rne((q[k,n] - z[k/g, n]) * s[k/g, n]), T = fp16 or bf16.
template <typename T>
__global__ void __launch_bounds__(256) awq_dequant_kernel(
    T* __restrict__ w_out, const uint32_t* __restrict__ qweight,
    const uint32_t* __restrict__ qzeros, const __half* __restrict__ scales, int K, int words_n,
    int group) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(K) * words_n;
  if (idx >= total) return;
  const int k = static_cast<int>(idx / words_n);
  const int j = static_cast<int>(idx - static_cast<int64_t>(k) * words_n);
  const int gi = k / group;
  const uint32_t w = __ldg(qweight + idx);
  const uint32_t zw = __ldg(qzeros + static_cast<int64_t>(gi) * words_n + j);
  const uint4 s = __ldg(reinterpret_cast<const uint4*>(scales + (static_cast<int64_t>(gi) * words_n + j) * 8));
  uint32_t qb[4], zb[4];
  awq_word_biased<T>(w, qb);
  awq_word_biased<T>(zw, zb);
  uint4 out;
  out.x = awq_dq<T>(qb[0], zb[0], awq_scale2<T>(s.x));
  out.y = awq_dq<T>(qb[1], zb[1], awq_scale2<T>(s.y));
  out.z = awq_dq<T>(qb[2], zb[2], awq_scale2<T>(s.z));
  out.w = awq_dq<T>(qb[3], zb[3], awq_scale2<T>(s.w));
  reinterpret_cast<uint4*>(w_out)[idx] = out;
}

}  // namespace lmrs
