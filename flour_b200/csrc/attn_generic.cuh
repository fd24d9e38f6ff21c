// Generic paged attention: any element type, any head_dim <= 256, any block_size <= 1024,
// any n_rep, any number of query tokens per sequence. One CTA per (query token, query head).
//
// This is the per-row form of backend::cpu::paged_attention (src/backend/cpu.rs:57-112): the
// sequence's KV is walked block by block in logical order (KvCache::gather_blocks,
// src/models/common/cache.rs:83-96) and folded with the same online softmax, in f32, with
// accurate expf, so f32 pools match the reference to ~1e-6. The bf16/f16 fast paths live in
// decode_sm100.cuh / prefill_sm100.cuh; this kernel serves f32 pools and shapes those do not
// cover (e.g. the reference's unit-test shapes: head_dim 4, block sizes 2-4).
#pragma once

#include "fa_common.cuh"

namespace fa {

struct GenericParams {
  const void *q;
  void *out;
  const void *k_cache;
  const void *v_cache;
  const int32_t *cu_seqlens_q;  // [num_seqs+1]; nullptr means one query per sequence (decode)
  const int32_t *context_lens;
  const int32_t *block_tables;
  int32_t max_blocks_per_seq;
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t n_rep;
  int32_t head_dim;
  int32_t block_size;
  int32_t num_blocks;
  int32_t total_q;
  float scale;
};

constexpr int kGenericThreads = 128;
constexpr int kGenericMaxDim = 256;

template <typename T>
__global__ void __launch_bounds__(kGenericThreads) generic_attn_kernel(const GenericParams p) {
  extern __shared__ float gsm[];
  float *qs = gsm;                    // [head_dim]
  float *sc = gsm + kGenericMaxDim;   // [block_size]
  const int qi = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = p.head_dim, BS = p.block_size;
  const size_t orow = (size_t(qi) * p.num_heads + h) * D;
  T *out = static_cast<T *>(p.out);

  // Locate the sequence of query token qi.
  int s, i, sq;
  if (p.cu_seqlens_q == nullptr) {
    s = qi; i = 0; sq = 1;
  } else {
    int lo = 0, hi = p.num_seqs;  // last s with cu[s] <= qi
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.cu_seqlens_q[mid] <= qi) lo = mid; else hi = mid;
    }
    s = lo;
    const int q0 = p.cu_seqlens_q[s], q1 = p.cu_seqlens_q[s + 1];
    if (q0 > qi || q1 <= qi || q1 > p.total_q) {
      if (tid == 0) report(FA_DEVERR_SEQLEN);
      for (int x = tid; x < D; x += kGenericThreads) out[orow + x] = Elem<T>::from_f(0.f);
      return;
    }
    i = qi - q0; sq = q1 - q0;
  }
  const int L = p.context_lens[s];
  if (L < sq || int64_t(L) > int64_t(p.max_blocks_per_seq) * BS) {
    if (tid == 0) report(FA_DEVERR_CONTEXT);
    for (int x = tid; x < D; x += kGenericThreads) out[orow + x] = Elem<T>::from_f(0.f);
    return;
  }
  const int offset = L - sq;  // cpu.rs:68
  const int kh = h / p.n_rep;
  const T *qp = static_cast<const T *>(p.q) + orow;
  for (int x = tid; x < D; x += kGenericThreads) qs[x] = Elem<T>::to_f(qp[x]);
  __syncthreads();

  const T *kc = static_cast<const T *>(p.k_cache);
  const T *vc = static_cast<const T *>(p.v_cache);
  float acc0 = 0.f, acc1 = 0.f;  // dims tid and tid + 128
  float m = neg_inf(), l = 0.f;
  const int nb = (L + BS - 1) / BS;
  const int32_t *table = p.block_tables + size_t(s) * p.max_blocks_per_seq;
  bool bad_id = false;
  for (int b = 0; b < nb; ++b) {
    int id = table[b];
    if (uint32_t(id) >= uint32_t(p.num_blocks)) { bad_id = true; id = 0; }
    const int kv_start = b * BS;
    const int bn = min(BS, L - kv_start);
    const size_t base = (size_t(id) * p.num_kv_heads + kh) * BS * size_t(D);
    // Scores of this block (cpu.rs:84-94): one warp per key row, lanes over head_dim.
    for (int j = warp; j < bn; j += kGenericThreads / 32) {
      const T *kr = kc + base + size_t(j) * D;
      float dot = 0.f;
      for (int x = lane; x < D; x += 32) dot += qs[x] * Elem<T>::to_f(kr[x]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (lane == 0) sc[j] = (kv_start + j > offset + i) ? neg_inf() : dot * p.scale;
    }
    __syncthreads();
    // Fold (cpu.rs:96-105); every thread evaluates the same scalar recurrence.
    float bmax = neg_inf();
    for (int j = 0; j < bn; ++j) bmax = fmaxf(bmax, sc[j]);
    const float new_max = fmaxf(m, bmax);
    const float corr = expf(m - new_max);
    float psum = 0.f, a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < bn; ++j) {
      const float pj = expf(sc[j] - new_max);
      psum += pj;
      const T *vr = vc + base + size_t(j) * D;
      if (tid < D) a0 += pj * Elem<T>::to_f(vr[tid]);
      if (tid + kGenericThreads < D) a1 += pj * Elem<T>::to_f(vr[tid + kGenericThreads]);
    }
    l = l * corr + psum;
    acc0 = acc0 * corr + a0;
    acc1 = acc1 * corr + a1;
    m = new_max;
    __syncthreads();
  }
  if (bad_id && tid == 0) report(FA_DEVERR_BLOCK_ID);
  // cpu.rs:111: acc / running_sum, cast to the query dtype.
  if (tid < D) out[orow + tid] = Elem<T>::from_f(acc0 / l);
  if (tid + kGenericThreads < D) out[orow + tid + kGenericThreads] = Elem<T>::from_f(acc1 / l);
}

}  // namespace fa
